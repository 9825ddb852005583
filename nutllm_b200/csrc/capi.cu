/* C ABI of libnutcuda.so (include/nutllm_cuda.h).
 *
 * Owns the device images of quantised matrices and models, the per-sequence
 * KV cache and decode state, and drives the token loop on one CUDA stream
 * per model.  Every failure is reported as a nut_status plus a thread-local
 * "component: reason" message; argument checks raise the same classes, in
 * the same order, as the reference's decode_quantized_token
 * (src/quant_model.cpp:161-172) and prefill_quantized (:212-213).
 */
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/nutllm_cuda.h"
#include "decode_mk.h"
#include "prefill.h"
#include "kernels.h"
#include "kernels_tc.h"

namespace {

thread_local std::string g_error;

} // namespace

void nut::set_last_error(const std::string &message) { g_error = message; }

namespace {
std::atomic<uint64_t> g_launches{0};
}

void nut::count_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
uint64_t nut::launches_so_far() { return g_launches.load(std::memory_order_relaxed); }
void nut::uncount_launches(uint64_t n) { g_launches.fetch_sub(n, std::memory_order_relaxed); }

namespace {

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

/* Waits for the uploads and memsets issued on the legacy default stream.
 * Host-to-device copies from pageable memory and device memsets return
 * before they complete, and the library's own streams are non-blocking
 * (they do not wait for the legacy stream), so every object is settled
 * before its handle is returned. */
void settle_uploads() { cuda_check(cudaStreamSynchronize(nullptr), "finish uploads"); }

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

void check_view(const nut_qmatrix_view &v, int64_t rows, int64_t cols, int type,
                const char *name) {
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

/* Packs reference storage into fragment tiles on the device. */
nut::TileMatrix upload_tiles(const nut_qmatrix_view &v, int order = nut::kRowMajor) {
    nut::TileMatrix t;
    t.shape = nut::TileShape::of(v.rows, v.cols, v.type, order);
    std::vector<uint8_t> data(t.shape.data_bytes());
    std::vector<uint16_t> scales(t.shape.scale_count());
    nut::pack_tiles(t.shape, v.data, v.scales, data.data(), scales.data());
    t.data = dev_alloc<uint8_t>(data.size(), "alloc tiles");
    t.scales = dev_alloc<uint16_t>(scales.size(), "alloc tile scales");
    cuda_check(cudaMemcpy(t.data, data.data(), data.size(), cudaMemcpyHostToDevice),
               "copy tiles");
    cuda_check(cudaMemcpy(t.scales, scales.data(), scales.size() * 2,
                          cudaMemcpyHostToDevice),
               "copy tile scales");
    return t;
}

void release(nut::TileMatrix &t) {
    dev_free(t.data);
    dev_free(t.scales);
    t.data = nullptr;
    t.scales = nullptr;
}

/* Stacks matrices with equal cols (reference storage, cols % 32 == 0, so
 * no block spans two of them) and packs the result into fragment tiles. */
nut::TileMatrix upload_stacked(std::initializer_list<const nut_qmatrix_view *> parts) {
    const nut_qmatrix_view &first = **parts.begin();
    int64_t rows = 0;
    for (const nut_qmatrix_view *v : parts)
        rows += v->rows;
    nut_qmatrix_view all = first;
    all.rows = rows;
    const int64_t cols = first.cols;
    std::vector<uint8_t> data;
    std::vector<uint16_t> scales;
    for (const nut_qmatrix_view *v : parts) {
        const size_t n = size_t(v->rows * cols);
        const size_t nd = first.type == NUT_QUANT_INT8 ? n : n / 2;
        data.insert(data.end(), v->data, v->data + nd);
        scales.insert(scales.end(), v->scales, v->scales + n / 32);
    }
    all.data = data.data();
    all.scales = scales.data();
    return upload_tiles(all);
}

/* Gate and up projections interleaved in groups of 8 rows, so one 16-row
 * tile holds gate and up rows of the same 8 hidden units. */
nut::TileMatrix upload_gate_up(const nut_qmatrix_view &gate, const nut_qmatrix_view &up) {
    const int64_t ffn = gate.rows, cols = gate.cols;
    const size_t row_bytes = size_t(gate.type == NUT_QUANT_INT8 ? cols : cols / 2);
    const size_t row_scales = size_t(cols / 32);
    std::vector<uint8_t> data(2 * size_t(ffn) * row_bytes);
    std::vector<uint16_t> scales(2 * size_t(ffn) * row_scales);
    for (int64_t r = 0; r < 2 * ffn; r++) {
        const int64_t group = r / 16, within = r % 16;
        const bool is_up = within >= 8;
        const int64_t src = group * 8 + (within % 8);
        const nut_qmatrix_view &v = is_up ? up : gate;
        std::copy(v.data + src * row_bytes, v.data + (src + 1) * row_bytes,
                  data.begin() + r * row_bytes);
        std::copy(v.scales + src * row_scales, v.scales + (src + 1) * row_scales,
                  scales.begin() + r * row_scales);
    }
    nut_qmatrix_view all = gate;
    all.rows = 2 * ffn;
    all.data = data.data();
    all.scales = scales.data();
    return upload_tiles(all);
}

/* Device-side error word -> status (bounded waits that gave up). */
void check_device_error(int *error_dev, cudaStream_t stream) {
    int code = 0;
    cuda_check(cudaMemcpyAsync(&code, error_dev, sizeof code, cudaMemcpyDeviceToHost,
                               stream),
               "read error word");
    cuda_check(cudaStreamSynchronize(stream), "synchronize");
    if (code != 0) {
        cudaMemsetAsync(error_dev, 0, sizeof(int), stream);
        cudaStreamSynchronize(stream);
        raise(NUT_DEVICE_TIMEOUT,
              "device: bounded wait gave up (code " + std::to_string(code) + ")");
    }
}

} // namespace

struct nut_qmatrix {
    int device = 0;
    int64_t rows = 0, cols = 0;
    int type = 0;
    bool tiled = false;
    nut::DevQMatrix m;  /* reference layout (blocks spanning rows) */
    nut::TileMatrix t;  /* fragment tiles (cols % 32 == 0) */
    float *x = nullptr, *y = nullptr; /* staging for host-buffer calls */
    int *error = nullptr;
    cudaStream_t stream = nullptr;
    /* prefill GEMM state: the dequantised fp16 copy of the matrix
     * [row_tiles * 16][blocks * 32] (made on first use) and the fp16
     * activation buffer */
    uint16_t *wbf = nullptr, *xbf = nullptr;
    size_t xbf_cap = 0;
    ~nut_qmatrix() {
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        release(m);
        release(t);
        dev_free(x);
        dev_free(y);
        dev_free(error);
        dev_free(wbf);
        dev_free(xbf);
    }
    void launch(const float *xd, float *yd, cudaStream_t s) {
        if (tiled) {
            cuda_check(nut::launch_qmatvec_tc(t, xd, yd, error, nut::kDefaultWaitNs, s),
                       "qmatvec launch");
            return;
        }
        nut::QSegs q{};
        q.seg[0] = seg(m, yd, 0);
        q.count = 1;
        q.cols = int(cols);
        q.type = type;
        nut::launch_qmatvec(q, xd, nullptr, s);
        cuda_check(cudaGetLastError(), "qmatvec launch");
    }
};

struct DevLayer {
    nut::DevQMatrix q, k, v, o, gate, up, down;
    float *attention_norm = nullptr, *ffn_norm = nullptr;
    /* fp32-weight models: q, k, v, o, gate, up, down as fp32 [out][in] */
    float *f[7] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
};

struct nut_model {
    int device = 0;
    nut_config cfg{};
    int64_t kv_heads = 0;
    int type = 0;
    bool tied = false;
    bool f32 = false; /* fp32 projections (ModelWeights), per-phase path only */
    float *embeddings = nullptr, *final_norm = nullptr, *lm_head = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr; /* [max_seq][hd/2] */
    std::vector<DevLayer> layers;
    uint64_t storage_bytes = 0;
    cudaStream_t stream = nullptr;
    /* persistent-kernel image (block-aligned shapes) */
    bool mk = false;
    int sms = 0;
    std::vector<nut::MkLayer> mk_layers;
    nut::MkLayerPtrs *mk_ptrs = nullptr;
    float *attn_norms = nullptr, *ffn_norms = nullptr; /* [layers][dim] */
    /* batched prefill: prompts of at least prefill_min tokens (0 = never)
     * run layer by layer as GEMMs over fp16 copies of the weights, made on
     * first use */
    int64_t prefill_min = 64;
    struct F16Layer {
        uint16_t *qkv = nullptr, *wo = nullptr, *gu = nullptr, *down = nullptr;
    };
    std::vector<F16Layer> f16w;
    int *gemm_error = nullptr;
    /* creation in steps (nut_model_begin / add_layer / finish) */
    bool building = false;
    int64_t added = 0;
    std::vector<nut::MkLayerPtrs> build_ptrs;
    std::vector<float> build_an, build_fn;
    ~nut_model() {
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        for (auto &b : f16w)
            dev_free(b.qkv), dev_free(b.wo), dev_free(b.gu), dev_free(b.down);
        dev_free(gemm_error);
        for (auto &l : mk_layers) {
            release(l.qkv), release(l.wo), release(l.gu), release(l.down);
        }
        dev_free(mk_ptrs), dev_free(attn_norms), dev_free(ffn_norms);
        for (auto &l : layers) {
            release(l.q), release(l.k), release(l.v), release(l.o);
            release(l.gate), release(l.up), release(l.down);
            dev_free(l.attention_norm), dev_free(l.ffn_norm);
            for (float *p : l.f)
                dev_free(p);
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
    float *x = nullptr, *tmp = nullptr; /* [dim] fp32-weight path scratch */
    unsigned long long *argmax_key = nullptr;
    int32_t *ids = nullptr; /* [max_seq] generated ids */
    bool has_hidden = false;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    /* persistent-kernel state */
    nut::Tagged *tagged = nullptr; /* q | k | v of the current token */
    float *mk_acc = nullptr;       /* [kAccSlots][dim] residual accumulators */
    unsigned int *mk_cnt = nullptr; /* [kAccSlots] step counters */
    size_t tagged_count = 0;
    unsigned long long *mk_keys = nullptr; /* [max_seq] */
    unsigned int *mk_done = nullptr;       /* [max_seq] */
    int32_t *mk_prompt = nullptr;          /* [max_seq] */
    int *mk_error = nullptr;
    unsigned long long *mk_stamps = nullptr; /* [3] */
    float *mk_logits = nullptr;
    size_t mk_logits_cap = 0;
    /* batched prefill scratch, rows for pf_cap tokens */
    float *pf_h = nullptr, *pf_qkv = nullptr, *pf_gu = nullptr;
    uint16_t *pf_x = nullptr, *pf_ctx = nullptr, *pf_act = nullptr;
    int32_t *pf_tok = nullptr;
    int64_t pf_cap = 0;
    void free_prefill() {
        dev_free(pf_h), dev_free(pf_qkv), dev_free(pf_gu), dev_free(pf_x), dev_free(pf_ctx);
        dev_free(pf_act), dev_free(pf_tok);
        pf_h = pf_qkv = pf_gu = nullptr;
        pf_x = pf_ctx = pf_act = nullptr;
        pf_tok = nullptr;
        pf_cap = 0;
    }
    ~nut_kv() {
        if (model)
            cudaStreamSynchronize(model->stream);
        dev_free(keys), dev_free(values), dev_free(hidden), dev_free(q);
        dev_free(k), dev_free(v), dev_free(ctx), dev_free(gate), dev_free(up);
        dev_free(x), dev_free(tmp);
        dev_free(logits), dev_free(argmax_key), dev_free(ids);
        dev_free(tagged), dev_free(mk_keys), dev_free(mk_done), dev_free(mk_prompt);
        dev_free(mk_acc), dev_free(mk_cnt);
        free_prefill();
        dev_free(mk_error), dev_free(mk_stamps), dev_free(mk_logits);
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
    if (m->f32) {
        /* decode_token over fp32 weights (src/kvcache.cpp:265-284,
         * decoder_layer_step :143-171) */
        const int kvd = KVH * hd, ffn = int(c.ffn_dim);
        auto mv = [&](const float *w, const float *xin, float *y, int rows, int cols) {
            cuda_check(nut::matvec_f32(w, xin, y, rows, cols, s), "fp32 projection");
        };
        for (int l = 0; l < int(c.layers); l++) {
            const DevLayer &w = m->layers[size_t(l)];
            cuda_check(nut::rmsnorm_vec(kv->hidden, w.attention_norm, kv->x, dim, s),
                       "rmsnorm");
            mv(w.f[0], kv->x, kv->q, dim, dim);
            mv(w.f[1], kv->x, kv->k, kvd, dim);
            mv(w.f[2], kv->x, kv->v, kvd, dim);
            nut::launch_rope_store(kv->q, kv->k, kv->v, kv->keys, kv->values, m->rope_cos,
                                   m->rope_sin, pos, l, H, KVH, hd, S, s);
            nut::launch_attention(kv->q, kv->keys, kv->values, kv->ctx, pos, l, H, KVH, hd, S,
                                  s);
            mv(w.f[3], kv->ctx, kv->tmp, dim, dim);
            cuda_check(nut::add_vec(kv->hidden, kv->tmp, dim, s), "residual");
            cuda_check(nut::rmsnorm_vec(kv->hidden, w.ffn_norm, kv->x, dim, s), "rmsnorm");
            mv(w.f[4], kv->x, kv->gate, ffn, dim);
            mv(w.f[5], kv->x, kv->up, ffn, dim);
            nut::launch_swiglu(kv->gate, kv->up, ffn, s);
            mv(w.f[6], kv->gate, kv->tmp, dim, ffn);
            cuda_check(nut::add_vec(kv->hidden, kv->tmp, dim, s), "residual");
        }
        cuda_check(cudaGetLastError(), "decode launch");
        kv->length++;
        kv->has_hidden = true;
        return;
    }
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

const char *token_range_message(const nut_model *m) {
    return m->f32 ? "kv cache: token id out of range" : "quantized decode: token out of range";
}

void check_decode_args(nut_model *m, nut_kv *kv, int64_t token) {
    if (m == nullptr || kv == nullptr)
        raise(NUT_INVALID_ARGUMENT, "quantized decode: null handle");
    if (kv->model != m)
        raise(NUT_INVALID_ARGUMENT, "quantized decode: cache configuration mismatch");
    /* the fp32 path keeps decode_token's messages (src/kvcache.cpp:35-41,
     * 265-276) */
    if (token < 0 || token >= m->cfg.vocab_size)
        raise(NUT_OUT_OF_RANGE, token_range_message(m));
    if (kv->length >= m->cfg.max_seq)
        raise(NUT_LENGTH_ERROR,
              m->f32 ? "kv cache: context is full" : "quantized decode: context is full");
}

void sync(nut_model *m) { cuda_check(cudaStreamSynchronize(m->stream), "synchronize"); }

/* One persistent-kernel launch: decode tokens[0..n_prompt) then greedy
 * tokens up to n_tokens decode passes in total, starting at start_pos.
 * Logits (and argmax ids) are produced after passes lfrom..lto.  Leaves
 * the last hidden vector in kv->hidden. */
void run_mk(nut_model *m, nut_kv *kv, const int32_t *tokens, int64_t n_prompt,
            int64_t n_tokens, int64_t start_pos, int64_t lfrom, int64_t lto,
            float *logits_host, int32_t *ids_host, nut_generation_stats *stats) {
    const nut_config &c = m->cfg;
    cudaStream_t s = m->stream;
    const int64_t nlog = lto >= lfrom ? lto - lfrom + 1 : 0;
    if (logits_host != nullptr && nlog > 0 &&
        kv->mk_logits_cap < size_t(nlog) * size_t(c.vocab_size)) {
        cuda_check(cudaStreamSynchronize(s), "synchronize");
        dev_free(kv->mk_logits);
        kv->mk_logits_cap = size_t(nlog) * size_t(c.vocab_size);
        kv->mk_logits = dev_alloc<float>(kv->mk_logits_cap, "alloc logits");
    }
    cuda_check(cudaMemcpyAsync(kv->mk_prompt, tokens, size_t(n_prompt) * 4,
                               cudaMemcpyHostToDevice, s),
               "copy prompt");
    cuda_check(cudaMemsetAsync(kv->mk_acc, 0, size_t(nut::kAccSlots) * c.dim * 4, s),
               "clear accumulators");
    cuda_check(cudaMemsetAsync(kv->mk_cnt, 0, size_t(nut::kAccSlots) * 4, s), "clear counters");
    cuda_check(cudaMemsetAsync(kv->tagged, 0, kv->tagged_count * sizeof(nut::Tagged), s),
               "clear tags");
    cuda_check(cudaMemsetAsync(kv->mk_keys, 0, size_t(n_tokens) * 8, s), "clear keys");
    cuda_check(cudaMemsetAsync(kv->mk_done, 0, size_t(n_tokens) * 4, s), "clear counts");
    cuda_check(cudaMemsetAsync(kv->mk_error, 0, sizeof(int), s), "clear error");
    cuda_check(cudaMemsetAsync(kv->mk_stamps, 0, 3 * 8, s), "clear stamps");
    const int dim = int(c.dim), kvd = int(m->kv_heads * c.head_dim), ffn = int(c.ffn_dim);
    nut::MkParams p{};
    p.layers = int(c.layers);
    p.dim = dim;
    p.kvd = kvd;
    p.heads = int(c.heads);
    p.kv_heads = int(m->kv_heads);
    p.hd = int(c.head_dim);
    p.ffn = ffn;
    p.vocab = int(c.vocab_size);
    p.max_seq = int(c.max_seq);
    const nut::MkLayer &L0 = m->mk_layers[0];
    p.nb_dim = int(L0.qkv.shape.blocks);
    p.nb_ffn = int(L0.down.shape.blocks);
    p.rt_qkv = int(L0.qkv.shape.row_tiles);
    p.rt_wo = int(L0.wo.shape.row_tiles);
    p.rt_gu = int(L0.gu.shape.row_tiles);
    p.rt_down = int(L0.down.shape.row_tiles);
    p.layer = m->mk_ptrs;
    p.attn_norm = m->attn_norms;
    p.ffn_norm = m->ffn_norms;
    p.final_norm = m->final_norm;
    p.lm_head = m->output_weights();
    p.emb = m->embeddings;
    p.rope_cos = m->rope_cos;
    p.rope_sin = m->rope_sin;
    p.kcache = kv->keys;
    p.vcache = kv->values;
    p.qkv = kv->tagged;
    p.hacc = kv->mk_acc;
    p.hidden_out = kv->hidden;
    p.cnt = kv->mk_cnt;
    p.wo_pairs = int(L0.wo.shape.blocks / 2);
    p.cpp = std::max(1, std::min(m->sms / p.wo_pairs, p.rt_wo));
    p.count_aw = p.wo_pairs * p.cpp;
    p.nbf = int(c.ffn_dim / 32);
    p.count_gd = m->sms;
    p.rt_down_pairs = int(L0.down.shape.row_tiles / 2);
    p.gd_unit = nut::ffn_units_per_block(p.rt_down_pairs);
    p.gd_total = p.nbf * p.gd_unit;
    p.act = kv->tagged + dim + 2 * kvd;
    p.xchg = p.act + ffn;
    p.prompt = kv->mk_prompt;
    p.n_prompt = int(n_prompt);
    p.n_tokens = int(n_tokens);
    p.start_pos = int(start_pos);
    p.logits_from = nlog > 0 ? int(lfrom) : 1 << 30;
    p.logits_to = nlog > 0 ? int(lto) : -1;
    p.keys = kv->mk_keys;
    p.done = kv->mk_done;
    p.logits = logits_host != nullptr && nlog > 0 ? kv->mk_logits : nullptr;
    p.error = kv->mk_error;
    p.stamps = kv->mk_stamps;
    p.limit_ns = nut::kDefaultWaitNs;
    /* NUTLLM_TRACE_FILE: record per-CTA phase timestamps and append them
     * to that file (tracing aid; off by default) */
    const char *trace_file = std::getenv("NUTLLM_TRACE_FILE");
    unsigned long long *trace = nullptr;
    const int stride = int(n_tokens * (3 * c.layers + 1));
    if (trace_file != nullptr) {
        trace = dev_alloc<unsigned long long>(size_t(m->sms) * stride * nut::kTraceWords,
                                              "alloc trace");
        cuda_check(cudaMemsetAsync(trace, 0, size_t(m->sms) * stride * nut::kTraceWords * 8, s),
                   "clear trace");
        p.trace = trace;
        p.trace_stride = stride;
    }
    cuda_check(nut::launch_decode_mk(p, m->type, m->sms, s), "persistent kernel launch");
    if (trace != nullptr) {
        std::vector<unsigned long long> host(size_t(m->sms) * stride * nut::kTraceWords);
        cuda_check(cudaMemcpyAsync(host.data(), trace, host.size() * 8, cudaMemcpyDeviceToHost,
                                   s),
                   "copy trace");
        cuda_check(cudaStreamSynchronize(s), "synchronize");
        dev_free(trace);
        if (FILE *f = std::fopen(trace_file, "ab")) {
            const int32_t hdr[4] = {m->sms, stride, int32_t(n_tokens),
                                    int32_t(c.layers) | (nut::kTraceWords << 16)};
            std::fwrite(hdr, sizeof hdr, 1, f);
            std::fwrite(host.data(), 8, host.size(), f);
            std::fclose(f);
        }
    }
    std::vector<unsigned long long> keys(size_t(nlog > 0 ? nlog : 0));
    if (ids_host != nullptr && nlog > 0)
        cuda_check(cudaMemcpyAsync(keys.data(), kv->mk_keys + lfrom, size_t(nlog) * 8,
                                   cudaMemcpyDeviceToHost, s),
                   "copy ids");
    if (p.logits != nullptr)
        cuda_check(cudaMemcpyAsync(logits_host, kv->mk_logits,
                                   size_t(nlog) * size_t(c.vocab_size) * 4,
                                   cudaMemcpyDeviceToHost, s),
                   "copy logits");
    unsigned long long st[3] = {0, 0, 0};
    cuda_check(cudaMemcpyAsync(st, kv->mk_stamps, sizeof st, cudaMemcpyDeviceToHost, s),
               "copy stamps");
    check_device_error(kv->mk_error, s);
    for (size_t k = 0; k < keys.size(); k++)
        ids_host[k] = int32_t(~uint32_t(keys[k] & 0xffffffffull));
    kv->length = start_pos + n_tokens;
    kv->has_hidden = true;
    if (stats != nullptr) {
        const double total = st[2] > st[0] ? double(st[2] - st[0]) * 1e-9 : 0.0;
        const double pre = st[1] > st[0] ? double(st[1] - st[0]) * 1e-9 : total;
        stats->prefill_seconds = pre;
        stats->decode_seconds = total - pre;
    }
}

/* fp16 copies of every layer's weights for the prefill GEMMs. */
void ensure_f16(nut_model *m) {
    if (!m->f16w.empty())
        return;
    auto make = [&](const nut::TileMatrix &t) {
        const size_t n = size_t(t.shape.row_tiles * 16) * size_t(t.shape.blocks * 32);
        uint16_t *p = dev_alloc<uint16_t>(n, "alloc fp16 weights");
        cuda_check(nut::dequant_tiles_f16(t, p, m->stream), "dequantize");
        return p;
    };
    for (const nut::MkLayer &L : m->mk_layers) {
        nut_model::F16Layer b;
        b.qkv = make(L.qkv);
        b.wo = make(L.wo);
        b.gu = make(L.gu);
        b.down = make(L.down);
        m->f16w.push_back(b);
    }
    m->gemm_error = dev_alloc<int>(1, "alloc error word");
    cuda_check(cudaMemsetAsync(m->gemm_error, 0, sizeof(int), m->stream), "clear error word");
}

/* The prompt through every layer as one batch (positions 0 .. n - 1):
 * per layer rmsnorm -> [q;k;v] GEMM -> RoPE + KV append -> causal attention
 * -> h += Wo ctx (GEMM) -> rmsnorm -> gate/up GEMM -> SwiGLU -> h += Wdown a
 * (GEMM).  Leaves the last token's hidden vector in kv->hidden. */
void prefill_batched(nut_model *m, nut_kv *kv, const int32_t *tokens, int64_t n) {
    const nut_config &c = m->cfg;
    cudaStream_t s = m->stream;
    const int dim = int(c.dim), kvd = int(m->kv_heads * c.head_dim), ffn = int(c.ffn_dim);
    const nut::MkLayer &L0 = m->mk_layers[0];
    const int kp_dim = int(L0.qkv.shape.blocks * 32), kp_ffn = int(L0.down.shape.blocks * 32);
    const int nqkv = dim + 2 * kvd, M = int(n);
    ensure_f16(m);
    if (kv->pf_cap < n) {
        cuda_check(cudaStreamSynchronize(s), "synchronize");
        kv->free_prefill();
        const size_t r = size_t(n);
        kv->pf_h = dev_alloc<float>(r * dim, "alloc prefill rows");
        kv->pf_qkv = dev_alloc<float>(r * nqkv, "alloc prefill rows");
        kv->pf_gu = dev_alloc<float>(r * 2 * ffn, "alloc prefill rows");
        kv->pf_x = dev_alloc<uint16_t>(r * kp_dim, "alloc prefill rows");
        kv->pf_ctx = dev_alloc<uint16_t>(r * kp_dim, "alloc prefill rows");
        kv->pf_act = dev_alloc<uint16_t>(r * kp_ffn, "alloc prefill rows");
        kv->pf_tok = dev_alloc<int32_t>(r, "alloc prefill tokens");
        kv->pf_cap = n;
    }
    cuda_check(cudaMemcpyAsync(kv->pf_tok, tokens, size_t(n) * 4, cudaMemcpyHostToDevice, s),
               "copy prompt");
    cuda_check(nut::gather_rows(m->embeddings, kv->pf_tok, M, dim, int(c.vocab_size), kv->pf_h, s),
               "embed");
    auto gemm = [&](const uint16_t *a, const nut::TileMatrix &t, const uint16_t *w, int N,
                    int K, float *y, bool acc) {
        cuda_check(nut::gemm_f16(a, M, w, N, int(t.shape.row_tiles * 16), K, y, N,
                                  m->gemm_error, nut::kDefaultWaitNs, s, acc),
                   "prefill gemm");
    };
    for (int64_t l = 0; l < c.layers; l++) {
        const nut::MkLayer &L = m->mk_layers[size_t(l)];
        const nut_model::F16Layer &B = m->f16w[size_t(l)];
        cuda_check(nut::rmsnorm_rows(kv->pf_h, m->attn_norms + l * dim, M, dim, kp_dim, kv->pf_x, s),
                   "rmsnorm");
        gemm(kv->pf_x, L.qkv, B.qkv, nqkv, kp_dim, kv->pf_qkv, false);
        cuda_check(nut::rope_kv_rows(kv->pf_qkv, M, nqkv, 0, m->rope_cos, m->rope_sin,
                                     int(c.heads), int(m->kv_heads), int(c.head_dim), dim, kvd,
                                     kv->keys, kv->values, int(l), int(c.max_seq), s),
                   "rope");
        cuda_check(nut::attention_prefill(kv->pf_qkv, M, 1, nqkv, 0, 1, 0, kv->keys, kv->values,
                                          int(l), int(c.heads), int(m->kv_heads),
                                          int(c.head_dim), int(c.max_seq), kp_dim, kv->pf_ctx,
                                          false, s),
                   "attention");
        cuda_check(nut::zero_tail(kv->pf_ctx, M, dim, kp_dim, s), "attention");
        gemm(kv->pf_ctx, L.wo, B.wo, dim, kp_dim, kv->pf_h, true);
        cuda_check(nut::rmsnorm_rows(kv->pf_h, m->ffn_norms + l * dim, M, dim, kp_dim, kv->pf_x, s),
                   "rmsnorm");
        gemm(kv->pf_x, L.gu, B.gu, 2 * ffn, kp_dim, kv->pf_gu, false);
        cuda_check(nut::swiglu_rows(kv->pf_gu, M, ffn, kp_ffn, kv->pf_act, s), "swiglu");
        gemm(kv->pf_act, L.down, B.down, dim, kp_ffn, kv->pf_h, true);
    }
    cuda_check(cudaMemcpyAsync(kv->hidden, kv->pf_h + size_t(n - 1) * dim, size_t(dim) * 4,
                               cudaMemcpyDeviceToDevice, s),
               "copy hidden");
    check_device_error(m->gemm_error, s);
    kv->length = n;
    kv->has_hidden = true;
}

/* RoPE table with the reference's exact fp32 values: frequency
 * 10000^(-pair/d) and cos/sin in double, rounded to fp32
 * (src/quant_model.cpp:26-37). */
void upload_rope(nut_model *m) {
    const nut_config &c = m->cfg;
    const size_t half = size_t(c.head_dim / 2), S = size_t(c.max_seq);
    std::vector<float> cs(S * half), sn(S * half);
    for (size_t p = 0; p < S; p++)
        for (size_t j = 0; j < half; j++) {
            const double f = std::pow(10000.0, -double(2 * j) / double(c.head_dim));
            cs[p * half + j] = float(std::cos(double(p) * f));
            sn[p * half + j] = float(std::sin(double(p) * f));
        }
    m->rope_cos = dev_alloc<float>(S * half, "alloc rope");
    m->rope_sin = dev_alloc<float>(S * half, "alloc rope");
    cuda_check(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice),
               "copy rope");
    cuda_check(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice),
               "copy rope");
}

bool use_batched_prefill(const nut_model *m, int64_t n) {
    const nut_config &c = m->cfg;
    const int kvd = int(m->kv_heads * c.head_dim), nqkv = int(c.dim) + 2 * kvd;
    return m->mk && m->prefill_min > 0 && n >= m->prefill_min &&
           nut::attention_prefill_supported(int(c.heads), int(m->kv_heads), int(c.head_dim),
                                            nqkv);
}

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
        if (view->data == nullptr || view->scales == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matrix: null storage");
        if (view->block_size != 32)
            raise(NUT_INVALID_ARGUMENT, "quantized matrix: block size must be 32");
        DeviceScope scope(device);
        auto q = std::make_unique<nut_qmatrix>();
        q->device = device;
        q->rows = view->rows;
        q->cols = view->cols;
        q->type = view->type;
        q->tiled = view->cols % 32 == 0;
        if (q->tiled)
            q->t = upload_tiles(*view);
        else
            q->m = upload(*view, view->rows, view->cols, view->type, "matrix");
        q->error = dev_alloc<int>(1, "alloc error word");
        cuda_check(cudaMemset(q->error, 0, sizeof(int)), "clear error word");
        q->x = dev_alloc<float>(size_t(view->cols), "alloc x");
        q->y = dev_alloc<float>(size_t(view->rows), "alloc y");
        cuda_check(cudaStreamCreateWithFlags(&q->stream, cudaStreamNonBlocking),
                   "create stream");
        settle_uploads();
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
        if (matrix->tiled) {
            const nut::TileShape &sh = matrix->t.shape;
            std::vector<uint8_t> td(sh.data_bytes());
            std::vector<uint16_t> ts(sh.scale_count());
            cuda_check(cudaMemcpy(td.data(), matrix->t.data, td.size(),
                                  cudaMemcpyDeviceToHost),
                       "download tiles");
            cuda_check(cudaMemcpy(ts.data(), matrix->t.scales, ts.size() * 2,
                                  cudaMemcpyDeviceToHost),
                       "download tile scales");
            nut::unpack_tiles(sh, td.data(), ts.data(), data, scales);
            return;
        }
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
        matrix->launch(x_device, y_device, static_cast<cudaStream_t>(stream));
    });
}

nut_status nut_qmatrix_gemm(nut_qmatrix *matrix, const float *x_device, int64_t tokens,
                            float *y_device, void *stream) {
    return guarded([&] {
        if (matrix == nullptr || x_device == nullptr || y_device == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized gemm: null pointer");
        if (tokens <= 0 || tokens > (int64_t(1) << 24))
            raise(NUT_INVALID_ARGUMENT, "quantized gemm: invalid token count");
        if (!matrix->tiled)
            raise(NUT_INVALID_ARGUMENT,
                  "quantized gemm: columns must be a multiple of the block size");
        DeviceScope scope(matrix->device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const nut::TileShape &sh = matrix->t.shape;
        const int64_t kp = sh.blocks * 32, n_alloc = sh.row_tiles * 16;
        if (matrix->wbf == nullptr) {
            matrix->wbf = dev_alloc<uint16_t>(size_t(n_alloc * kp), "alloc fp16 weights");
            cuda_check(nut::dequant_tiles_f16(matrix->t, matrix->wbf, s), "dequantize");
        }
        const size_t need = size_t(tokens * kp);
        if (matrix->xbf_cap < need) {
            cuda_check(cudaStreamSynchronize(s), "synchronize");
            dev_free(matrix->xbf);
            matrix->xbf = dev_alloc<uint16_t>(need, "alloc fp16 activations");
            matrix->xbf_cap = need;
        }
        cuda_check(nut::round_f16(x_device, int(tokens), int(matrix->cols), int(kp),
                                   matrix->xbf, s),
                   "round activations");
        cuda_check(nut::gemm_f16(matrix->xbf, int(tokens), matrix->wbf, int(matrix->rows),
                                  int(n_alloc), int(kp), y_device, int(matrix->rows),
                                  matrix->error, nut::kDefaultWaitNs, s),
                   "gemm launch");
    });
}

nut_status nut_matmul_f32(const float *a, const float *b, float *c, int64_t m, int64_t k,
                          int64_t n, void *stream) {
    return guarded([&] {
        if (a == nullptr || b == nullptr || c == nullptr)
            raise(NUT_INVALID_ARGUMENT, "threaded matmul: null pointer");
        if (m <= 0 || k <= 0 || n <= 0 || m > INT32_MAX || k > INT32_MAX || n > INT32_MAX)
            raise(NUT_INVALID_ARGUMENT, "threaded matmul: shape mismatch");
        cuda_check(nut::matmul_f32(a, b, c, int(m), int(k), int(n),
                                   static_cast<cudaStream_t>(stream)),
                   "matmul launch");
    });
}

nut_status nut_matvec_f32(const float *matrix, const float *vector, float *output,
                          int64_t rows, int64_t cols, void *stream) {
    return guarded([&] {
        if (matrix == nullptr || vector == nullptr || output == nullptr)
            raise(NUT_INVALID_ARGUMENT, "threaded matvec: null pointer");
        if (rows <= 0 || cols <= 0 || rows > INT32_MAX || cols > INT32_MAX)
            raise(NUT_INVALID_ARGUMENT, "threaded matvec: invalid shape");
        cuda_check(nut::matvec_f32(matrix, vector, output, int(rows), int(cols),
                                   static_cast<cudaStream_t>(stream)),
                   "matvec launch");
    });
}

nut_status nut_qmatrix_error(nut_qmatrix *matrix) {
    return guarded([&] {
        if (matrix == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matrix: null handle");
        DeviceScope scope(matrix->device);
        check_device_error(matrix->error, matrix->stream);
    });
}

nut_status nut_qmatvec(nut_qmatrix *matrix, const float *x, float *y) {
    return guarded([&] {
        if (matrix == nullptr || x == nullptr || y == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized matvec: null pointer");
        DeviceScope scope(matrix->device);
        const size_t cols = size_t(matrix->cols), rows = size_t(matrix->rows);
        cuda_check(cudaMemcpyAsync(matrix->x, x, cols * 4, cudaMemcpyHostToDevice,
                                   matrix->stream),
                   "copy x");
        matrix->launch(matrix->x, matrix->y, matrix->stream);
        cuda_check(cudaMemcpyAsync(y, matrix->y, rows * 4, cudaMemcpyDeviceToHost,
                                   matrix->stream),
                   "copy y");
        check_device_error(matrix->error, matrix->stream);
    });
}

/* Model creation in three steps (nut_model_create runs all three): the
 * fp32 tensors and the shape checks, then one layer at a time (its
 * projections packed into tiles and uploaded), then the tables of the
 * persistent kernel and the RoPE rows.  A loader can quantise layer l + 1
 * on the host while layer l is added. */
void model_begin(nut_model &mm, const nut_model_view *view, int device) {
    if (view == nullptr)
        raise(NUT_INVALID_ARGUMENT, "model: null argument");
    const nut_config &c = view->config;
    validate_config(c);
    if (view->quant_type != NUT_QUANT_INT8 && view->quant_type != NUT_QUANT_INT4)
        raise(NUT_INVALID_ARGUMENT, "model: unknown quant type");
    if (view->embeddings == nullptr || view->final_norm == nullptr ||
        (!view->tied_embeddings && view->lm_head == nullptr))
        raise(NUT_INVALID_ARGUMENT, "model: null fp32 tensor");
    nut_model *m = &mm;
    m->device = device;
    m->cfg = c;
    m->kv_heads = c.kv_heads == 0 ? c.heads : c.kv_heads;
    m->type = view->quant_type;
    m->tied = view->tied_embeddings != 0;
    cuda_check(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "create stream");
    const size_t dim = size_t(c.dim), V = size_t(c.vocab_size);
    const int64_t kvd = m->kv_heads * c.head_dim;
    m->storage_bytes = (V * dim + dim + (m->tied ? 0 : V * dim)) * 4;
    m->embeddings = dev_alloc<float>(V * dim, "alloc embeddings");
    cuda_check(cudaMemcpy(m->embeddings, view->embeddings, V * dim * 4, cudaMemcpyHostToDevice),
               "copy embeddings");
    m->final_norm = dev_alloc<float>(dim, "alloc final norm");
    cuda_check(cudaMemcpy(m->final_norm, view->final_norm, dim * 4, cudaMemcpyHostToDevice),
               "copy final norm");
    if (!m->tied) {
        m->lm_head = dev_alloc<float>(V * dim, "alloc lm_head");
        cuda_check(cudaMemcpy(m->lm_head, view->lm_head, V * dim * 4, cudaMemcpyHostToDevice),
                   "copy lm_head");
    }
    int max_smem = 0;
    cuda_check(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, device),
               "device attribute");
    cuda_check(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device),
               "device attribute");
    int coop = 0;
    cuda_check(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device),
               "device attribute");
    m->mk = coop != 0 && nut::mk_supported(int(c.dim), int(c.ffn_dim), int(kvd),
                                           int(c.head_dim), int(c.heads), view->quant_type,
                                           max_smem, m->sms);
    m->building = true;
    m->added = 0;
    m->build_ptrs.clear();
    m->build_an.clear();
    m->build_fn.clear();
}

void model_add_layer(nut_model &mm, const nut_layer_view &lv) {
    nut_model *m = &mm;
    const nut_config &c = m->cfg;
    if (!m->building || m->added >= c.layers)
        raise(NUT_INVALID_ARGUMENT, "quantized decode: layer count mismatch");
    if (lv.attention_norm == nullptr || lv.ffn_norm == nullptr)
        raise(NUT_INVALID_ARGUMENT, "model: null norm weights");
    const size_t dim = size_t(c.dim);
    const int64_t kvd = m->kv_heads * c.head_dim;
    const int t = m->type;
    if (m->mk) {
        check_view(lv.query, c.dim, c.dim, t, "query");
        check_view(lv.key, kvd, c.dim, t, "key");
        check_view(lv.value, kvd, c.dim, t, "value");
        check_view(lv.output, c.dim, c.dim, t, "output");
        check_view(lv.gate, c.ffn_dim, c.dim, t, "gate");
        check_view(lv.up, c.ffn_dim, c.dim, t, "up");
        check_view(lv.down, c.dim, c.ffn_dim, t, "down");
        m->mk_layers.emplace_back();
        nut::MkLayer &d = m->mk_layers.back();
        d.qkv = upload_stacked({&lv.query, &lv.key, &lv.value});
        d.wo = upload_tiles(lv.output, nut::kPairColumn);
        d.gu = upload_gate_up(lv.gate, lv.up);
        d.down = upload_tiles(lv.down, nut::kBlockColumn);
        m->build_ptrs.push_back({d.qkv.data, d.wo.data, d.gu.data, d.down.data, d.qkv.scales,
                                 d.wo.scales, d.gu.scales, d.down.scales});
        for (const nut_qmatrix_view *q : {&lv.query, &lv.key, &lv.value, &lv.output, &lv.gate,
                                          &lv.up, &lv.down}) {
            const size_t n = size_t(q->rows * q->cols);
            m->storage_bytes += (t == NUT_QUANT_INT8 ? n : (n + 1) / 2) + (n + 31) / 32 * 2;
        }
        m->build_an.insert(m->build_an.end(), lv.attention_norm, lv.attention_norm + dim);
        m->build_fn.insert(m->build_fn.end(), lv.ffn_norm, lv.ffn_norm + dim);
    } else {
        m->layers.emplace_back();
        DevLayer &d = m->layers.back();
        d.q = upload(lv.query, c.dim, c.dim, t, "query");
        d.k = upload(lv.key, kvd, c.dim, t, "key");
        d.v = upload(lv.value, kvd, c.dim, t, "value");
        d.o = upload(lv.output, c.dim, c.dim, t, "output");
        d.gate = upload(lv.gate, c.ffn_dim, c.dim, t, "gate");
        d.up = upload(lv.up, c.ffn_dim, c.dim, t, "up");
        d.down = upload(lv.down, c.dim, c.ffn_dim, t, "down");
        for (const nut::DevQMatrix *q : {&d.q, &d.k, &d.v, &d.o, &d.gate, &d.up, &d.down})
            m->storage_bytes += q->data_bytes() + q->scale_count() * 2;
        d.attention_norm = dev_alloc<float>(dim, "alloc norm");
        d.ffn_norm = dev_alloc<float>(dim, "alloc norm");
        cuda_check(cudaMemcpy(d.attention_norm, lv.attention_norm, dim * 4,
                              cudaMemcpyHostToDevice),
                   "copy norm");
        cuda_check(cudaMemcpy(d.ffn_norm, lv.ffn_norm, dim * 4, cudaMemcpyHostToDevice),
                   "copy norm");
    }
    m->storage_bytes += 2 * dim * 4;
    m->added++;
}

void model_finish(nut_model &mm) {
    nut_model *m = &mm;
    if (!m->building || m->added != m->cfg.layers)
        raise(NUT_INVALID_ARGUMENT, "quantized decode: layer count mismatch");
    if (m->mk) {
        const auto &ptrs = m->build_ptrs;
        m->mk_ptrs = dev_alloc<nut::MkLayerPtrs>(ptrs.size(), "alloc layer table");
        cuda_check(cudaMemcpy(m->mk_ptrs, ptrs.data(), ptrs.size() * sizeof(ptrs[0]),
                              cudaMemcpyHostToDevice),
                   "copy layer table");
        m->attn_norms = dev_alloc<float>(m->build_an.size(), "alloc norms");
        m->ffn_norms = dev_alloc<float>(m->build_fn.size(), "alloc norms");
        cuda_check(cudaMemcpy(m->attn_norms, m->build_an.data(), m->build_an.size() * 4,
                              cudaMemcpyHostToDevice),
                   "copy norms");
        cuda_check(cudaMemcpy(m->ffn_norms, m->build_fn.data(), m->build_fn.size() * 4,
                              cudaMemcpyHostToDevice),
                   "copy norms");
    }
    m->build_ptrs = {};
    m->build_an = {};
    m->build_fn = {};
    upload_rope(m);
    settle_uploads();
    m->building = false;
}

nut_status nut_model_create(const nut_model_view *view, int device,
                            nut_model **out) {
    return guarded([&] {
        if (view == nullptr || out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        validate_config(view->config);
        if (view->n_layers != view->config.layers || view->layers == nullptr)
            raise(NUT_INVALID_ARGUMENT, "quantized decode: layer count mismatch");
        DeviceScope scope(device);
        auto m = std::make_unique<nut_model>();
        model_begin(*m, view, device);
        for (int64_t l = 0; l < view->n_layers; l++)
            model_add_layer(*m, view->layers[l]);
        model_finish(*m);
        *out = m.release();
    });
}

nut_status nut_model_begin(const nut_model_view *view, int device, nut_model **out) {
    return guarded([&] {
        if (out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        DeviceScope scope(device);
        auto m = std::make_unique<nut_model>();
        model_begin(*m, view, device);
        *out = m.release();
    });
}

nut_status nut_model_add_layer(nut_model *model, const nut_layer_view *layer) {
    return guarded([&] {
        if (model == nullptr || layer == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        DeviceScope scope(model->device);
        model_add_layer(*model, *layer);
    });
}

nut_status nut_model_finish(nut_model *model) {
    return guarded([&] {
        if (model == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        DeviceScope scope(model->device);
        model_finish(*model);
    });
}

nut_status nut_model_create_f32(const nut_model_f32_view *view, int device, nut_model **out) {
    return guarded([&] {
        if (view == nullptr || out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        const nut_config &c = view->config;
        validate_config(c);
        if (view->n_layers != c.layers || view->layers == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: layer count mismatch");
        if (view->embeddings == nullptr || view->final_norm == nullptr ||
            (!view->tied_embeddings && view->lm_head == nullptr))
            raise(NUT_INVALID_ARGUMENT, "model: null fp32 tensor");
        DeviceScope scope(device);
        auto m = std::make_unique<nut_model>();
        m->device = device;
        m->cfg = c;
        m->kv_heads = c.kv_heads == 0 ? c.heads : c.kv_heads;
        m->type = -1;
        m->f32 = true;
        m->tied = view->tied_embeddings != 0;
        m->prefill_min = 0; /* the fp32 path has no GEMM prefill */
        cuda_check(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking),
                   "create stream");
        const size_t dim = size_t(c.dim), V = size_t(c.vocab_size), ffn = size_t(c.ffn_dim);
        const size_t kvd = size_t(m->kv_heads * c.head_dim);
        uint64_t bytes = 0;
        auto up = [&](const float *src, size_t n, const char *what) {
            if (src == nullptr)
                raise(NUT_INVALID_ARGUMENT, "model: null fp32 tensor");
            float *p = dev_alloc<float>(n, what);
            cuda_check(cudaMemcpy(p, src, n * 4, cudaMemcpyHostToDevice), what);
            bytes += n * 4;
            return p;
        };
        m->embeddings = up(view->embeddings, V * dim, "copy embeddings");
        m->final_norm = up(view->final_norm, dim, "copy final norm");
        if (!m->tied)
            m->lm_head = up(view->lm_head, V * dim, "copy lm_head");
        for (int64_t l = 0; l < c.layers; l++) {
            const nut_layer_f32_view &lv = view->layers[l];
            m->layers.emplace_back();
            DevLayer &d = m->layers.back();
            const float *src[7] = {lv.query, lv.key, lv.value, lv.output, lv.gate, lv.up,
                                   lv.down};
            const size_t n[7] = {dim * dim, kvd * dim, kvd * dim, dim * dim, ffn * dim,
                                 ffn * dim, dim * ffn};
            for (int j = 0; j < 7; j++)
                d.f[j] = up(src[j], n[j], "copy fp32 weights");
            d.attention_norm = up(lv.attention_norm, dim, "copy norm");
            d.ffn_norm = up(lv.ffn_norm, dim, "copy norm");
        }
        m->storage_bytes = bytes;
        upload_rope(m.get());
        settle_uploads();
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

nut_status nut_model_stream(const nut_model *model, void **stream) {
    return guarded([&] {
        if (model == nullptr || stream == nullptr)
            raise(NUT_INVALID_ARGUMENT, "model: null argument");
        *stream = static_cast<void *>(model->stream);
    });
}

nut_status nut_model_set_prefill_threshold(nut_model *model, int64_t min_tokens) {
    return guarded([&] {
        if (model == nullptr || min_tokens < 0)
            raise(NUT_INVALID_ARGUMENT, "model: invalid prefill threshold");
        model->prefill_min = min_tokens;
    });
}

nut_status nut_launch_count(uint64_t *count) {
    if (count == nullptr) {
        g_error = "launch count: null argument";
        return NUT_INVALID_ARGUMENT;
    }
    *count = g_launches.load(std::memory_order_relaxed);
    return NUT_OK;
}

nut_status nut_kv_create(nut_model *model, nut_kv **out) {
    return guarded([&] {
        if (model == nullptr || out == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        if (model->building)
            raise(NUT_INVALID_ARGUMENT, "kv cache: model creation not finished");
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
        kv->x = dev_alloc<float>(size_t(c.dim), "alloc scratch");
        kv->tmp = dev_alloc<float>(size_t(c.dim), "alloc scratch");
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
        if (model->mk) {
            /* q | k | v, the SwiGLU outputs, and one partial attention
             * state (hd + 2 elements) per CTA */
            kv->tagged_count = size_t(c.dim) + 2 * kvd + size_t(c.ffn_dim) +
                               size_t(model->sms) * size_t(c.head_dim + 2);
            kv->mk_acc = dev_alloc<float>(size_t(nut::kAccSlots) * c.dim, "alloc accumulators");
            kv->mk_cnt = dev_alloc<unsigned int>(nut::kAccSlots, "alloc step counters");
            kv->tagged = dev_alloc<nut::Tagged>(kv->tagged_count, "alloc tagged");
            kv->mk_keys = dev_alloc<unsigned long long>(size_t(c.max_seq), "alloc keys");
            kv->mk_done = dev_alloc<unsigned int>(size_t(c.max_seq), "alloc counts");
            kv->mk_prompt = dev_alloc<int32_t>(size_t(c.max_seq), "alloc prompt");
            kv->mk_error = dev_alloc<int>(1, "alloc error word");
            kv->mk_stamps = dev_alloc<unsigned long long>(3, "alloc stamps");
        }
        settle_uploads();
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

nut_status nut_kv_write(nut_kv *kv, int64_t layer, int64_t position, const float *keys,
                        const float *values) {
    return guarded([&] {
        if (kv == nullptr || keys == nullptr || values == nullptr)
            raise(NUT_INVALID_ARGUMENT, "kv cache: null argument");
        const nut_model *m = kv->model;
        const nut_config &c = m->cfg;
        if (layer < 0 || layer >= c.layers || position < 0 || position >= c.max_seq)
            raise(NUT_OUT_OF_RANGE, "kv cache: store out of range");
        DeviceScope scope(m->device);
        const int64_t hd = c.head_dim;
        for (int64_t h = 0; h < m->kv_heads; h++) {
            const size_t off = size_t(((layer * m->kv_heads + h) * c.max_seq + position) * hd);
            cuda_check(cudaMemcpyAsync(kv->keys + off, keys + h * hd, size_t(hd) * 4,
                                       cudaMemcpyHostToDevice, m->stream),
                       "store key");
            cuda_check(cudaMemcpyAsync(kv->values + off, values + h * hd, size_t(hd) * 4,
                                       cudaMemcpyHostToDevice, m->stream),
                       "store value");
        }
        cuda_check(cudaStreamSynchronize(m->stream), "synchronize");
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
        if (model->mk) {
            const int32_t t = token;
            run_mk(model, kv, &t, 1, 1, kv->length, 1, 0, nullptr, nullptr, nullptr);
        } else {
            enqueue_decode(model, kv, token, 0);
        }
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
        for (int64_t i = 0; i < n; i++)
            if (tokens[i] < 0 || tokens[i] >= model->cfg.vocab_size)
                raise(NUT_OUT_OF_RANGE, token_range_message(model));
        if (use_batched_prefill(model, n)) {
            prefill_batched(model, kv, tokens, n);
        } else if (model->mk) {
            run_mk(model, kv, tokens, n, n, 0, 1, 0, nullptr, nullptr, nullptr);
        } else {
            for (int64_t i = 0; i < n; i++) {
                check_decode_args(model, kv, tokens[i]);
                enqueue_decode(model, kv, tokens[i], 0);
            }
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
                raise(NUT_OUT_OF_RANGE, token_range_message(model));
        DeviceScope scope(model->device);
        cudaStream_t s = model->stream;
        kv->length = 0;
        kv->has_hidden = false;
        if (model->mk) {
            /* one launch: the prompt, then every greedy step (logits and
             * argmax after passes n-1 .. n+steps-2; the last pass decodes
             * the last chosen token, as the reference loop does) */
            const int64_t steps = std::min<int64_t>(max_tokens, c.max_seq - n);
            std::vector<int32_t> chosen(size_t(std::max<int64_t>(steps, 1)));
            if (use_batched_prefill(model, n)) {
                /* the prompt as one batch, the first token from its last
                 * hidden vector, then the persistent loop from position n */
                cuda_check(cudaEventRecord(kv->ev[0], s), "event");
                prefill_batched(model, kv, prompt, n);
                cuda_check(cudaEventRecord(kv->ev[1], s), "event");
                double dec = 0.0;
                if (steps > 0) {
                    enqueue_logits(model, kv);
                    unsigned long long key = 0;
                    cuda_check(cudaMemcpyAsync(&key, kv->argmax_key, sizeof key,
                                               cudaMemcpyDeviceToHost, s),
                               "copy argmax");
                    if (logits != nullptr)
                        cuda_check(cudaMemcpyAsync(logits, kv->logits, c.vocab_size * 4,
                                                   cudaMemcpyDeviceToHost, s),
                                   "copy logits");
                    cuda_check(cudaEventRecord(kv->ev[2], s), "event");
                    sync(model);
                    chosen[0] = int32_t(~uint32_t(key & 0xffffffffull));
                    nut_generation_stats st{};
                    run_mk(model, kv, chosen.data(), 1, steps, n, 0, steps - 2,
                           logits != nullptr ? logits + c.vocab_size : nullptr,
                           chosen.data() + 1, &st);
                    float head_ms = 0.0f;
                    cuda_check(cudaEventElapsedTime(&head_ms, kv->ev[1], kv->ev[2]), "elapsed");
                    dec = st.prefill_seconds + st.decode_seconds + double(head_ms) * 1e-3;
                }
                sync(model);
                float pre_ms = 0.0f;
                cuda_check(cudaEventElapsedTime(&pre_ms, kv->ev[0], kv->ev[1]), "elapsed");
                if (stats != nullptr) {
                    stats->prefill_seconds = double(pre_ms) * 1e-3;
                    stats->decode_seconds = dec;
                }
            } else {
                run_mk(model, kv, prompt, n, n + steps, 0, n - 1, n + steps - 2, logits,
                       chosen.data(), stats);
            }
            int64_t produced = steps;
            if (stop_at_eos) {
                for (int64_t k = 0; k < steps; k++)
                    if (chosen[size_t(k)] == c.eos_token) {
                        produced = k;
                        break;
                    }
                /* the reference decodes exactly the emitted tokens */
                kv->length = n + produced;
            }
            std::copy(chosen.begin(), chosen.begin() + produced, ids);
            if (n_generated != nullptr)
                *n_generated = produced;
            if (stats != nullptr) {
                stats->prefill_tokens = n;
                stats->generated_tokens = produced;
            }
            return;
        }
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
