/* Tensor-parallel batched decoder (nut_batch_* in nutllm_cuda.h).
 *
 * B independent sequences advance one token per step, all at the same
 * position.  Each of `world` ranks (one process per GPU) holds one shard
 * of every layer, as the survey of the reference's Llama decoder splits it
 * ([out][in] storage, src/llama2.cpp:374-396):
 *   column-parallel  Wq, Wk, Wv rows of this rank's heads (heads / world
 *                    query heads, kv_heads / world kv heads), Wgate and
 *                    Wup rows of its ffn / world hidden units;
 *   row-parallel     Wo columns of its heads, Wdown columns of its units,
 *                    whose partial outputs are summed over the ranks with
 *                    one NCCL all-reduce each per layer;
 *   vocabulary split the classifier rows [v0, v1), with the first-index
 *                    argmax combined by a 64-bit max all-reduce of
 *                    (value, ~index) keys.
 * Embeddings and norms are replicated.  A step is: rmsnorm rows -> [q;k;v]
 * GEMM -> RoPE + KV append -> attention -> Wo GEMM -> all-reduce ->
 * residual + rmsnorm -> gate/up GEMM -> SwiGLU -> Wdown GEMM -> all-reduce,
 * per layer, then the final norm, classifier GEMM and argmax.  The GEMMs
 * are the tcgen05 fp16 GEMM of gemm_tc.cu over dequantised (q * scale
 * rounded to fp16) weights; activations are rounded to fp16 per GEMM.
 * NCCL is resolved at run time (dlopen of libnccl.so.2), so the library
 * loads without it and shares the copy an embedding process already holds.
 */
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include "../../include/nutllm_cuda.h"
#include "batch.h"
#include "kernels.h"
#include "kernels_tc.h"
#include "prefill.h"

namespace {

struct Failure {
    nut_status status;
    std::string message;
};

[[noreturn]] void raise(nut_status s, const std::string &m) { throw Failure{s, m}; }

void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess)
        raise(NUT_RUNTIME_ERROR, std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

template <typename F> nut_status guarded(F &&body) {
    try {
        body();
        return NUT_OK;
    } catch (const Failure &f) {
        nut::set_last_error(f.message);
        return f.status;
    } catch (const std::bad_alloc &) {
        nut::set_last_error("nutllm: host allocation failed");
        return NUT_RUNTIME_ERROR;
    } catch (const std::exception &e) {
        nut::set_last_error(e.what());
        return NUT_RUNTIME_ERROR;
    }
}

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
    cuda_check(cudaMalloc(&p, (count == 0 ? 1 : count) * sizeof(T)), what);
    return static_cast<T *>(p);
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

/* ---- NCCL, resolved at run time ------------------------------------ */

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr)
            h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (h != nullptr) {
            api.get_unique_id =
                reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
            api.comm_init_rank =
                reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
            api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
            api.comm_destroy =
                reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
            api.error_string =
                reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        }
    }
    if (api.get_unique_id == nullptr || api.comm_init_rank == nullptr ||
        api.all_reduce == nullptr || api.comm_destroy == nullptr)
        raise(NUT_RUNTIME_ERROR, "tensor parallel: libnccl.so.2 not available");
    return api;
}

void nccl_check(ncclResult_t r, const char *what) {
    if (r != ncclSuccess) {
        const char *msg = nccl().error_string ? nccl().error_string(r) : "error";
        raise(NUT_RUNTIME_ERROR, std::string("nccl: ") + what + ": " + msg);
    }
}

/* ---- host dequantisation of a view slice into fp16 ------------------ */

float qvalue(const nut_qmatrix_view &v, int64_t r, int64_t c) {
    const int64_t i = r * v.cols + c;
    int q;
    if (v.type == NUT_QUANT_INT8) {
        q = int(int8_t(v.data[i]));
    } else {
        const int nib = (v.data[i / 2] >> ((i & 1) ? 4 : 0)) & 0xF;
        q = nib >= 8 ? nib - 16 : nib;
    }
    return float(q) * __half2float(__ushort_as_half(v.scales[i / 32]));
}

uint16_t to_f16(float v) {
    v = std::fmin(std::fmax(v, -65504.0f), 65504.0f);
    return __half_as_ushort(__float2half_rn(v));
}

} // namespace

struct nut_batch {
    int device = 0, rank = 0, world = 1, B = 0;
    nut_config cfg{};
    int kvh = 0;                 /* kv heads of the model */
    int heads_r = 0, kvh_r = 0, hd = 0, dim = 0, ffn_r = 0, vocab_r = 0, v0 = 0;
    int max_seq = 0, layers = 0, nqkv = 0;
    int kp_dim = 0, kp_ctx = 0, kp_ffn = 0;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;
    struct Layer {
        uint16_t *qkv = nullptr, *wo = nullptr, *gu = nullptr, *down = nullptr; /* fp16 */
        uint8_t *qkv4 = nullptr, *wo4 = nullptr, *gu4 = nullptr, *down4 = nullptr; /* INT4 */
        float *attn_norm = nullptr, *ffn_norm = nullptr;
    };
    bool q4 = false; /* projections as packed INT4 (gemm_q4) rather than fp16 copies */
    std::vector<Layer> L;
    float *emb = nullptr, *final_norm = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    uint16_t *lm = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
    float *h = nullptr, *part = nullptr, *qkv = nullptr, *gu = nullptr, *logits = nullptr;
    uint16_t *x16 = nullptr, *ctx16 = nullptr, *act16 = nullptr;
    unsigned long long *keys = nullptr;
    int32_t *ids = nullptr, *out = nullptr, *prompts = nullptr;
    int *pos = nullptr, *pstep = nullptr, *ostep = nullptr; /* device counters */
    int *gemm_error = nullptr;
    /* prefill rows (chunks of whole sequences, made on first use) */
    int pf_rows = 0;
    float *pf_h = nullptr, *pf_part = nullptr, *pf_qkv = nullptr, *pf_gu = nullptr;
    uint16_t *pf_x16 = nullptr, *pf_ctx16 = nullptr, *pf_act16 = nullptr;
    int prefill_min = 16; /* prompts of at least this many tokens: GEMM prefill */
    /* peer-memory all-reduce: this rank's area ([2][world][B dim] floats,
     * then [world][kArChunks] flags), the peers' areas (IPC mappings), the
     * per-chunk call counters and the error word */
    uint8_t *peer_area = nullptr;
    std::vector<void *> peer_open;
    float *recv_ptrs[8] = {};
    unsigned *flag_ptrs[8] = {};
    unsigned *ar_epochs = nullptr;
    int *ar_error = nullptr;
    bool peers = false;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    uint64_t weight_bytes = 0; /* fp16 weights + fp32 tensors this rank holds */
    /* one captured prompt pass and one captured decode pass (their
     * positions and counters live in device memory, so a replay serves
     * every step); built on first use */
    cudaGraphExec_t g_prompt = nullptr, g_decode = nullptr;
    int g_prompt_n = 0;
    uint64_t g_prompt_kernels = 0, g_decode_kernels = 0;

    ~nut_batch() {
        if (stream == nullptr)
            return; /* nothing was allocated (the stream is created first) */
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        if (stream)
            cudaStreamSynchronize(stream);
        for (Layer &l : L)
            for (void *p : {(void *)l.qkv, (void *)l.wo, (void *)l.gu, (void *)l.down,
                            (void *)l.qkv4, (void *)l.wo4, (void *)l.gu4, (void *)l.down4,
                            (void *)l.attn_norm, (void *)l.ffn_norm})
                if (p)
                    cudaFree(p);
        for (void *p : {(void *)pf_h, (void *)pf_part, (void *)pf_qkv, (void *)pf_gu,
                        (void *)pf_x16, (void *)pf_ctx16, (void *)pf_act16})
            if (p)
                cudaFree(p);
        for (void *p : peer_open)
            cudaIpcCloseMemHandle(p);
        for (void *p : {(void *)peer_area, (void *)ar_epochs, (void *)ar_error})
            if (p)
                cudaFree(p);
        for (void *p : {(void *)emb, (void *)final_norm, (void *)rope_cos, (void *)rope_sin,
                        (void *)lm, (void *)kcache, (void *)vcache, (void *)h, (void *)part,
                        (void *)qkv, (void *)gu, (void *)logits, (void *)x16, (void *)ctx16,
                        (void *)act16, (void *)keys, (void *)ids, (void *)out,
                        (void *)prompts, (void *)pos, (void *)pstep, (void *)ostep,
                        (void *)gemm_error})
            if (p)
                cudaFree(p);
        for (cudaEvent_t e : ev)
            if (e)
                cudaEventDestroy(e);
        if (g_prompt)
            cudaGraphExecDestroy(g_prompt);
        if (g_decode)
            cudaGraphExecDestroy(g_decode);
        if (comm)
            nccl().comm_destroy(comm);
        if (stream)
            cudaStreamDestroy(stream);
        cudaSetDevice(prev);
    }
};

namespace {

/* Shard shape of rank `rank` of `world` (checks the split points). */
void plan_shard(nut_batch &b, const nut_config &c, int rank, int world, int64_t batch) {
    const int64_t kvh = c.kv_heads == 0 ? c.heads : c.kv_heads;
    if (c.layers <= 0 || c.heads <= 0 || c.dim <= 0 || c.head_dim <= 0 || c.ffn_dim <= 0 ||
        c.vocab_size <= 0 || c.max_seq <= 0 || c.heads * c.head_dim != c.dim ||
        c.head_dim % 4 != 0 || kvh <= 0 || c.heads % kvh != 0)
        raise(NUT_INVALID_ARGUMENT, "model config: invalid dimensions");
    if (world <= 0 || rank < 0 || rank >= world)
        raise(NUT_INVALID_ARGUMENT, "tensor parallel: invalid rank");
    if (c.heads % world != 0 || kvh % world != 0 || c.ffn_dim % (32 * world) != 0 ||
        c.vocab_size < world)
        raise(NUT_INVALID_ARGUMENT,
              "tensor parallel: heads, kv heads and ffn blocks must split evenly");
    if (batch <= 0 || batch > 4096)
        raise(NUT_INVALID_ARGUMENT, "batch: invalid size");
    b.cfg = c;
    b.rank = rank;
    b.world = world;
    b.B = int(batch);
    b.kvh = int(kvh);
    b.hd = int(c.head_dim);
    b.dim = int(c.dim);
    b.layers = int(c.layers);
    b.max_seq = int(c.max_seq);
    b.heads_r = int(c.heads / world);
    b.kvh_r = int(kvh / world);
    b.ffn_r = int(c.ffn_dim / world);
    b.v0 = int(c.vocab_size * rank / world);
    b.vocab_r = int(c.vocab_size * (rank + 1) / world) - b.v0;
    b.nqkv = (b.heads_r + 2 * b.kvh_r) * b.hd;
    b.kp_dim = round_up(b.dim, 64);
    b.kp_ctx = round_up(b.heads_r * b.hd, 64);
    b.kp_ffn = round_up(b.ffn_r, 64);
}

void alloc_state(nut_batch &b) {
    const size_t B = size_t(b.B);
    cuda_check(cudaStreamCreateWithFlags(&b.stream, cudaStreamNonBlocking), "create stream");
    for (cudaEvent_t &e : b.ev)
        cuda_check(cudaEventCreate(&e), "create event");
    const size_t kv = size_t(b.layers) * B * b.kvh_r * size_t(b.max_seq) * b.hd;
    b.kcache = dev_alloc<float>(kv, "alloc kv cache");
    b.vcache = dev_alloc<float>(kv, "alloc kv cache");
    b.h = dev_alloc<float>(B * b.dim, "alloc rows");
    b.part = dev_alloc<float>(B * b.dim, "alloc rows");
    b.qkv = dev_alloc<float>(B * b.nqkv, "alloc rows");
    b.gu = dev_alloc<float>(B * 2 * b.ffn_r, "alloc rows");
    b.logits = dev_alloc<float>(B * b.vocab_r, "alloc rows");
    b.x16 = dev_alloc<uint16_t>(B * b.kp_dim, "alloc rows");
    b.ctx16 = dev_alloc<uint16_t>(B * b.kp_ctx, "alloc rows");
    b.act16 = dev_alloc<uint16_t>(B * b.kp_ffn, "alloc rows");
    b.keys = dev_alloc<unsigned long long>(B, "alloc keys");
    b.ids = dev_alloc<int32_t>(B, "alloc ids");
    b.out = dev_alloc<int32_t>(B * b.max_seq, "alloc ids");
    b.prompts = dev_alloc<int32_t>(B * b.max_seq, "alloc prompts");
    b.pos = dev_alloc<int>(1, "alloc counters");
    b.pstep = dev_alloc<int>(1, "alloc counters");
    b.ostep = dev_alloc<int>(1, "alloc counters");
    b.gemm_error = dev_alloc<int>(1, "alloc error word");
    cuda_check(cudaMemset(b.gemm_error, 0, sizeof(int)), "clear error word");
    /* GEMM outputs start at zero: each step's GEMMs add into them and their
     * consumers zero them again */
    cuda_check(cudaMemset(b.part, 0, B * b.dim * 4), "clear rows");
    cuda_check(cudaMemset(b.qkv, 0, B * b.nqkv * 4), "clear rows");
    cuda_check(cudaMemset(b.gu, 0, B * 2 * b.ffn_r * 4), "clear rows");
    cuda_check(cudaMemset(b.logits, 0, B * b.vocab_r * 4), "clear rows");
    cuda_check(cudaMemset(b.keys, 0, B * sizeof(unsigned long long)), "clear keys");
    /* RoPE table with the reference's fp32 values (frequency and angle in
     * double, rounded once; src/quant_model.cpp:26-37) */
    const size_t half = size_t(b.hd / 2), S = size_t(b.max_seq);
    std::vector<float> cs(S * half), sn(S * half);
    for (size_t p = 0; p < S; p++)
        for (size_t j = 0; j < half; j++) {
            const double f = std::pow(10000.0, -double(2 * j) / double(b.hd));
            cs[p * half + j] = float(std::cos(double(p) * f));
            sn[p * half + j] = float(std::sin(double(p) * f));
        }
    b.rope_cos = dev_alloc<float>(S * half, "alloc rope");
    b.rope_sin = dev_alloc<float>(S * half, "alloc rope");
    cuda_check(cudaMemcpy(b.rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice),
               "copy rope");
    cuda_check(cudaMemcpy(b.rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice),
               "copy rope");
    b.L.resize(size_t(b.layers));
}

uint16_t *upload_f16(const std::vector<uint16_t> &v, uint64_t &bytes) {
    uint16_t *p = dev_alloc<uint16_t>(v.size(), "alloc fp16 weights");
    cuda_check(cudaMemcpy(p, v.data(), v.size() * 2, cudaMemcpyHostToDevice), "copy weights");
    bytes += v.size() * 2;
    return p;
}

float *upload_f32(const float *src, size_t n, uint64_t &bytes) {
    float *p = dev_alloc<float>(n, "alloc fp32 tensor");
    cuda_check(cudaMemcpy(p, src, n * 4, cudaMemcpyHostToDevice), "copy fp32 tensor");
    bytes += n * 4;
    return p;
}

/* INT4 projections stay packed and are dequantised inside the GEMM
 * pipeline when NUTLLM_BATCH_Q4=1.  Off by default: that pipeline is
 * latency-bound at its 64-row stages (~0.58 us per 64-wide K block against
 * ~0.35 us for the fp16 copies), so the fp16 copies are faster today in
 * spite of 3.6x the weight bytes. */
bool use_q4() {
    const char *v = std::getenv("NUTLLM_BATCH_Q4");
    return v != nullptr && v[0] == '1';
}

/* This rank's shard of a host model (the reference's storage), dequantised
 * to fp16 on the host (or packed INT4, see use_q4). */
void load_view(nut_batch &b, const nut_model_view &v) {
    const nut_config &c = b.cfg;
    if (v.n_layers != c.layers || v.layers == nullptr || v.embeddings == nullptr ||
        v.final_norm == nullptr || (!v.tied_embeddings && v.lm_head == nullptr))
        raise(NUT_INVALID_ARGUMENT, "model: incomplete view");
    const int dim = b.dim, hd = b.hd;
    const int q0 = b.rank * b.heads_r * hd, k0 = b.rank * b.kvh_r * hd;
    const int kvd_r = b.kvh_r * hd, f0 = b.rank * b.ffn_r;
    /* packed INT4 needs whole quant blocks in every slice */
    b.q4 = v.quant_type == NUT_QUANT_INT4 && use_q4() && dim % 32 == 0 &&
           (b.heads_r * hd) % 32 == 0;
    /* the listed (matrix, row) pairs, columns [c0, c0 + n), as contiguous
     * INT4 storage packed for gemm_q4 */
    auto pack_rows = [&](const std::vector<std::pair<const nut_qmatrix_view *, int>> &rows,
                         int c0, int n, int K) {
        std::vector<uint8_t> data(rows.size() * size_t(n / 2));
        std::vector<uint16_t> sc(rows.size() * size_t(n / 32));
        for (size_t r = 0; r < rows.size(); r++) {
            const nut_qmatrix_view &m = *rows[r].first;
            const int64_t src = rows[r].second;
            std::memcpy(data.data() + r * (n / 2), m.data + (src * m.cols + c0) / 2, n / 2);
            std::memcpy(sc.data() + r * (n / 32), m.scales + (src * m.cols + c0) / 32,
                        (n / 32) * 2);
        }
        std::vector<uint8_t> packed(nut::q4_packed_bytes(int(rows.size()), K));
        nut::pack_q4(data.data(), sc.data(), int(rows.size()), n, K, packed.data());
        uint8_t *p = dev_alloc<uint8_t>(packed.size(), "alloc packed weights");
        cuda_check(cudaMemcpy(p, packed.data(), packed.size(), cudaMemcpyHostToDevice),
                   "copy packed weights");
        b.weight_bytes += packed.size();
        return p;
    };
    for (int l = 0; l < b.layers; l++) {
        const nut_layer_view &lv = v.layers[l];
        for (const nut_qmatrix_view *m : {&lv.query, &lv.key, &lv.value, &lv.output, &lv.gate,
                                          &lv.up, &lv.down})
            if (m->data == nullptr || m->scales == nullptr || m->block_size != 32 ||
                m->type != v.quant_type)
                raise(NUT_INVALID_ARGUMENT, "model: invalid matrix view");
        if (b.q4) {
            nut_batch::Layer &d = b.L[size_t(l)];
            std::vector<std::pair<const nut_qmatrix_view *, int>> rows;
            for (int r = 0; r < b.heads_r * hd; r++)
                rows.push_back({&lv.query, q0 + r});
            for (int r = 0; r < kvd_r; r++)
                rows.push_back({&lv.key, k0 + r});
            for (int r = 0; r < kvd_r; r++)
                rows.push_back({&lv.value, k0 + r});
            d.qkv4 = pack_rows(rows, 0, dim, b.kp_dim);
            rows.clear();
            for (int r = 0; r < dim; r++)
                rows.push_back({&lv.output, r});
            d.wo4 = pack_rows(rows, q0, b.heads_r * hd, b.kp_ctx);
            rows.clear();
            for (int r = 0; r < 2 * b.ffn_r; r++) {
                const int group = r / 16, within = r % 16;
                rows.push_back({within >= 8 ? &lv.up : &lv.gate, f0 + group * 8 + within % 8});
            }
            d.gu4 = pack_rows(rows, 0, dim, b.kp_dim);
            rows.clear();
            for (int r = 0; r < dim; r++)
                rows.push_back({&lv.down, r});
            d.down4 = pack_rows(rows, f0, b.ffn_r, b.kp_ffn);
            d.attn_norm = upload_f32(lv.attention_norm, size_t(dim), b.weight_bytes);
            d.ffn_norm = upload_f32(lv.ffn_norm, size_t(dim), b.weight_bytes);
            continue;
        }
        std::vector<uint16_t> qkv(size_t(b.nqkv) * b.kp_dim, 0);
        for (int r = 0; r < b.nqkv; r++) {
            const nut_qmatrix_view *m;
            int src;
            if (r < b.heads_r * hd) {
                m = &lv.query;
                src = q0 + r;
            } else if (r < b.heads_r * hd + kvd_r) {
                m = &lv.key;
                src = k0 + r - b.heads_r * hd;
            } else {
                m = &lv.value;
                src = k0 + r - b.heads_r * hd - kvd_r;
            }
            for (int k = 0; k < dim; k++)
                qkv[size_t(r) * b.kp_dim + k] = to_f16(qvalue(*m, src, k));
        }
        std::vector<uint16_t> wo(size_t(dim) * b.kp_ctx, 0);
        for (int r = 0; r < dim; r++)
            for (int k = 0; k < b.heads_r * hd; k++)
                wo[size_t(r) * b.kp_ctx + k] = to_f16(qvalue(lv.output, r, q0 + k));
        std::vector<uint16_t> gu(size_t(2 * b.ffn_r) * b.kp_dim, 0);
        for (int r = 0; r < 2 * b.ffn_r; r++) {
            const int group = r / 16, within = r % 16;
            const nut_qmatrix_view &m = within >= 8 ? lv.up : lv.gate;
            const int src = f0 + group * 8 + within % 8;
            for (int k = 0; k < dim; k++)
                gu[size_t(r) * b.kp_dim + k] = to_f16(qvalue(m, src, k));
        }
        std::vector<uint16_t> down(size_t(dim) * b.kp_ffn, 0);
        for (int r = 0; r < dim; r++)
            for (int k = 0; k < b.ffn_r; k++)
                down[size_t(r) * b.kp_ffn + k] = to_f16(qvalue(lv.down, r, f0 + k));
        nut_batch::Layer &d = b.L[size_t(l)];
        d.qkv = upload_f16(qkv, b.weight_bytes);
        d.wo = upload_f16(wo, b.weight_bytes);
        d.gu = upload_f16(gu, b.weight_bytes);
        d.down = upload_f16(down, b.weight_bytes);
        d.attn_norm = upload_f32(lv.attention_norm, size_t(dim), b.weight_bytes);
        d.ffn_norm = upload_f32(lv.ffn_norm, size_t(dim), b.weight_bytes);
    }
    b.emb = upload_f32(v.embeddings, size_t(c.vocab_size) * dim, b.weight_bytes);
    b.final_norm = upload_f32(v.final_norm, size_t(dim), b.weight_bytes);
    const float *cls = v.tied_embeddings ? v.embeddings : v.lm_head;
    std::vector<uint16_t> lm(size_t(b.vocab_r) * b.kp_dim, 0);
    for (int r = 0; r < b.vocab_r; r++)
        for (int k = 0; k < dim; k++)
            lm[size_t(r) * b.kp_dim + k] = to_f16(cls[size_t(b.v0 + r) * dim + k]);
    b.lm = upload_f16(lm, b.weight_bytes);
}

/* Seeded synthetic shard generated on the device: random INT4 block-32
 * projections (dequantised to fp16), N(0, 0.02) embeddings and classifier,
 * unit norm gains. */
void load_synthetic(nut_batch &b, uint64_t seed) {
    const int dim = b.dim;
    cudaStream_t s = b.stream;
    const float sigma = 0.02f;
    auto stream_id = [&](int layer, int which) {
        return uint64_t(layer) * 64 + uint64_t(which) * 8 + uint64_t(b.rank) + 1;
    };
    auto make = [&](int rows, int cols, int ld, uint64_t id) {
        uint16_t *p = dev_alloc<uint16_t>(size_t(rows) * ld, "alloc fp16 weights");
        cuda_check(nut::synth_int4_f16_dev(seed, id, sigma, rows, cols, ld, p, s), "synth");
        b.weight_bytes += size_t(rows) * ld * 2;
        return p;
    };
    auto make4 = [&](int rows, int cols, int K, uint64_t id) {
        const size_t bytes = nut::q4_packed_bytes(rows, K);
        uint8_t *p = dev_alloc<uint8_t>(bytes, "alloc packed weights");
        cuda_check(nut::synth_q4_packed_dev(seed, id, sigma, rows, cols, K, p, s), "synth");
        b.weight_bytes += bytes;
        return p;
    };
    b.q4 = use_q4();
    std::vector<float> ones(size_t(dim), 1.0f);
    for (int l = 0; l < b.layers; l++) {
        nut_batch::Layer &d = b.L[size_t(l)];
        if (b.q4) {
            d.qkv4 = make4(b.nqkv, dim, b.kp_dim, stream_id(l, 0));
            d.wo4 = make4(dim, b.heads_r * b.hd, b.kp_ctx, stream_id(l, 1));
            d.gu4 = make4(2 * b.ffn_r, dim, b.kp_dim, stream_id(l, 2));
            d.down4 = make4(dim, b.ffn_r, b.kp_ffn, stream_id(l, 3));
            d.attn_norm = upload_f32(ones.data(), size_t(dim), b.weight_bytes);
            d.ffn_norm = upload_f32(ones.data(), size_t(dim), b.weight_bytes);
            continue;
        }
        d.qkv = make(b.nqkv, dim, b.kp_dim, stream_id(l, 0));
        d.wo = make(dim, b.heads_r * b.hd, b.kp_ctx, stream_id(l, 1));
        d.gu = make(2 * b.ffn_r, dim, b.kp_dim, stream_id(l, 2));
        d.down = make(dim, b.ffn_r, b.kp_ffn, stream_id(l, 3));
        d.attn_norm = upload_f32(ones.data(), size_t(dim), b.weight_bytes);
        d.ffn_norm = upload_f32(ones.data(), size_t(dim), b.weight_bytes);
    }
    const size_t V = size_t(b.cfg.vocab_size);
    b.emb = dev_alloc<float>(V * dim, "alloc embeddings");
    cuda_check(nut::synth_normal_dev(seed, 1u << 20, sigma, b.emb, V * dim, s), "synth");
    b.weight_bytes += V * dim * 4;
    b.final_norm = upload_f32(ones.data(), size_t(dim), b.weight_bytes);
    float *cls = dev_alloc<float>(size_t(b.vocab_r) * dim, "alloc classifier");
    cuda_check(nut::synth_normal_dev(seed, (2u << 20) + uint64_t(b.rank), sigma, cls,
                                     size_t(b.vocab_r) * dim, s),
               "synth");
    b.lm = dev_alloc<uint16_t>(size_t(b.vocab_r) * b.kp_dim, "alloc classifier");
    cuda_check(nut::round_f16(cls, b.vocab_r, dim, b.kp_dim, b.lm, s), "round classifier");
    b.weight_bytes += size_t(b.vocab_r) * b.kp_dim * 2;
    cuda_check(cudaStreamSynchronize(s), "synthesise weights");
    cudaFree(cls);
}

/* y[B][N] += x w^T; y holds zeros (every consumer of a GEMM output zeroes
 * it once read), so the K dimension may be split over CTAs that add their
 * partial products. */
void gemm(nut_batch &b, const uint16_t *a, const uint16_t *w, int N, int K, float *y,
          int M = 0) {
    cuda_check(nut::gemm_f16(a, M > 0 ? M : b.B, w, N, N, K, y, N, b.gemm_error,
                             nut::kDefaultWaitNs, b.stream, true, 8),
               "batch gemm");
}

/* A projection: packed INT4 weights through gemm_q4, or the fp16 copy. */
void proj(nut_batch &b, const uint16_t *a, const uint16_t *w16, const uint8_t *w4, int N, int K,
          float *y, int M = 0) {
    if (b.q4)
        cuda_check(nut::gemm_q4(a, M > 0 ? M : b.B, w4, N, K, y, N, b.gemm_error,
                                nut::kDefaultWaitNs, b.stream, true, 8),
                   "batch gemm");
    else
        gemm(b, a, w16, N, K, y, M);
}

void all_reduce_sum(nut_batch &b, float *x, size_t n) {
    if (b.world == 1)
        return;
    if (b.peers)
        cuda_check(nut::peer_all_reduce(x, x, int(n), b.recv_ptrs, b.flag_ptrs, b.rank,
                                        b.world, b.ar_epochs, b.ar_error, nut::kDefaultWaitNs,
                                        b.stream),
                   "peer all-reduce");
    else
        nccl_check(nccl().all_reduce(x, x, n, ncclFloat32, ncclSum, b.comm, b.stream),
                   "all-reduce");
}

size_t peer_area_bytes(const nut_batch &b) {
    return size_t(2) * b.world * size_t(b.B) * b.dim * 4 +
           size_t(b.world) * nut::kArChunks * 4;
}

/* One forward pass of the batch: token ids in b.ids at position *b.pos,
 * every layer; the hidden rows stay in b.h with the last Wdown partial
 * (already summed over the ranks) in b.part. */
void forward(nut_batch &b) {
    cudaStream_t s = b.stream;
    const int B = b.B, dim = b.dim;
    cuda_check(nut::gather_rows(b.emb, b.ids, B, dim, int(b.cfg.vocab_size), b.h, s), "embed");
    for (int l = 0; l < b.layers; l++) {
        const nut_batch::Layer &L = b.L[size_t(l)];
        /* layer 0 starts from the embedding rows: the previous pass's
         * last Wdown partial is only cleared */
        cuda_check(nut::add_rmsnorm_rows(b.h, b.part, l > 0, L.attn_norm, B, dim, b.kp_dim,
                                         b.x16, s),
                   "rmsnorm");
        proj(b, b.x16, L.qkv, L.qkv4, b.nqkv, b.kp_dim, b.qkv);
        cuda_check(nut::rope_kv_batch(b.qkv, B, b.nqkv, b.pos, b.rope_cos, b.rope_sin,
                                      b.heads_r, b.kvh_r, b.hd, b.kcache, b.vcache, l,
                                      b.max_seq, s),
                   "rope");
        cuda_check(nut::attention_batch(b.qkv, B, b.nqkv, b.pos, b.kcache, b.vcache, l,
                                        b.heads_r, b.kvh_r, b.hd, b.max_seq, b.kp_ctx, b.ctx16,
                                        s),
                   "attention");
        proj(b, b.ctx16, L.wo, L.wo4, dim, b.kp_ctx, b.part);
        all_reduce_sum(b, b.part, size_t(B) * dim);
        cuda_check(nut::add_rmsnorm_rows(b.h, b.part, true, L.ffn_norm, B, dim, b.kp_dim,
                                         b.x16, s),
                   "rmsnorm");
        proj(b, b.x16, L.gu, L.gu4, 2 * b.ffn_r, b.kp_dim, b.gu);
        cuda_check(nut::swiglu_rows(b.gu, B, b.ffn_r, b.kp_ffn, b.act16, s, true), "swiglu");
        proj(b, b.act16, L.down, L.down4, dim, b.kp_ffn, b.part);
        all_reduce_sum(b, b.part, size_t(B) * dim);
    }
}

/* The prompts [B][n] through every layer as GEMMs over the rows of up to
 * kPrefillRows tokens (whole sequences per chunk): the same operations as
 * n passes of forward(), with RoPE, the KV append and causal attention per
 * sequence.  Leaves each sequence's last hidden row in b.h (and its last
 * Wdown partial, summed over the ranks, in b.part), the cache holding
 * positions 0 .. n - 1 and *pos = n - 1, as the n-th pass would. */
constexpr int kPrefillRows = 2048;

void prefill(nut_batch &b, int n) {
    cudaStream_t s = b.stream;
    const int dim = b.dim, chunk = std::max(1, std::min(b.B, kPrefillRows / n));
    const int rows = chunk * n;
    if (b.pf_rows < rows) {
        cuda_check(cudaStreamSynchronize(s), "synchronize");
        for (void *p : {(void *)b.pf_h, (void *)b.pf_part, (void *)b.pf_qkv, (void *)b.pf_gu,
                        (void *)b.pf_x16, (void *)b.pf_ctx16, (void *)b.pf_act16})
            if (p)
                cudaFree(p);
        const size_t R = size_t(rows);
        b.pf_h = dev_alloc<float>(R * dim, "alloc prefill rows");
        b.pf_part = dev_alloc<float>(R * dim, "alloc prefill rows");
        b.pf_qkv = dev_alloc<float>(R * b.nqkv, "alloc prefill rows");
        b.pf_gu = dev_alloc<float>(R * 2 * b.ffn_r, "alloc prefill rows");
        b.pf_x16 = dev_alloc<uint16_t>(R * b.kp_dim, "alloc prefill rows");
        b.pf_ctx16 = dev_alloc<uint16_t>(R * b.kp_ctx, "alloc prefill rows");
        b.pf_act16 = dev_alloc<uint16_t>(R * b.kp_ffn, "alloc prefill rows");
        /* GEMM outputs start at zero; their consumers zero them again */
        cuda_check(cudaMemsetAsync(b.pf_part, 0, R * dim * 4, s), "clear rows");
        cuda_check(cudaMemsetAsync(b.pf_qkv, 0, R * b.nqkv * 4, s), "clear rows");
        cuda_check(cudaMemsetAsync(b.pf_gu, 0, R * 2 * b.ffn_r * 4, s), "clear rows");
        b.pf_rows = rows;
    }
    for (int s0 = 0; s0 < b.B; s0 += chunk) {
        const int cs = std::min(chunk, b.B - s0), M = cs * n;
        cuda_check(nut::gather_rows(b.emb, b.prompts + size_t(s0) * n, M, dim,
                                    int(b.cfg.vocab_size), b.pf_h, s),
                   "embed");
        for (int l = 0; l < b.layers; l++) {
            const nut_batch::Layer &L = b.L[size_t(l)];
            cuda_check(nut::add_rmsnorm_rows(b.pf_h, b.pf_part, l > 0, L.attn_norm, M, dim,
                                             b.kp_dim, b.pf_x16, s),
                       "rmsnorm");
            proj(b, b.pf_x16, L.qkv, L.qkv4, b.nqkv, b.kp_dim, b.pf_qkv, M);
            cuda_check(nut::rope_kv_batch(b.pf_qkv, b.B, b.nqkv, b.pos, b.rope_cos, b.rope_sin,
                                          b.heads_r, b.kvh_r, b.hd, b.kcache, b.vcache, l,
                                          b.max_seq, s, M, n, s0),
                       "rope");
            cuda_check(nut::attention_prefill(b.pf_qkv, n, cs, b.nqkv, s0, b.B, 0, b.kcache,
                                              b.vcache, l, b.heads_r, b.kvh_r, b.hd, b.max_seq,
                                              b.kp_ctx, b.pf_ctx16, true, s),
                       "attention");
            proj(b, b.pf_ctx16, L.wo, L.wo4, dim, b.kp_ctx, b.pf_part, M);
            if (b.world > 1)
                nccl_check(nccl().all_reduce(b.pf_part, b.pf_part, size_t(M) * dim, ncclFloat32,
                                             ncclSum, b.comm, s),
                           "all-reduce");
            cuda_check(nut::add_rmsnorm_rows(b.pf_h, b.pf_part, true, L.ffn_norm, M, dim,
                                             b.kp_dim, b.pf_x16, s),
                       "rmsnorm");
            proj(b, b.pf_x16, L.gu, L.gu4, 2 * b.ffn_r, b.kp_dim, b.pf_gu, M);
            cuda_check(nut::swiglu_rows(b.pf_gu, M, b.ffn_r, b.kp_ffn, b.pf_act16, s, true),
                       "swiglu");
            proj(b, b.pf_act16, L.down, L.down4, dim, b.kp_ffn, b.pf_part, M);
            if (b.world > 1)
                nccl_check(nccl().all_reduce(b.pf_part, b.pf_part, size_t(M) * dim, ncclFloat32,
                                             ncclSum, b.comm, s),
                           "all-reduce");
        }
        /* each sequence's last row: hidden and its pending Wdown partial */
        const size_t pitch = size_t(n) * dim * 4, row = size_t(dim) * 4;
        cuda_check(cudaMemcpy2DAsync(b.h + size_t(s0) * dim, row,
                                     b.pf_h + size_t(n - 1) * dim, pitch, row, cs,
                                     cudaMemcpyDeviceToDevice, s),
                   "copy last rows");
        cuda_check(cudaMemcpy2DAsync(b.part + size_t(s0) * dim, row,
                                     b.pf_part + size_t(n - 1) * dim, pitch, row, cs,
                                     cudaMemcpyDeviceToDevice, s),
                   "copy last rows");
        /* the partials of the other rows are never added: clear them all */
        cuda_check(cudaMemsetAsync(b.pf_part, 0, size_t(M) * dim * 4, s), "clear rows");
    }
    const int last = n - 1;
    cuda_check(cudaMemcpyAsync(b.pos, &last, sizeof last, cudaMemcpyHostToDevice, s),
               "set position");
    cuda_check(cudaStreamSynchronize(s), "prefill"); /* `last` lives on this stack */
}

/* Final norm, this rank's classifier rows, and the global first-index
 * argmax into b.ids (and b.out[:, *ostep]). */
void head(nut_batch &b, bool keep_logits) {
    cudaStream_t s = b.stream;
    cuda_check(nut::add_rmsnorm_rows(b.h, b.part, true, b.final_norm, b.B, b.dim, b.kp_dim,
                                     b.x16, s),
               "final norm");
    gemm(b, b.x16, b.lm, b.vocab_r, b.kp_dim, b.logits);
    cuda_check(nut::argmax_keys(b.logits, b.B, b.vocab_r, b.v0, b.keys, !keep_logits, s),
               "argmax");
    if (b.world > 1)
        nccl_check(nccl().all_reduce(b.keys, b.keys, size_t(b.B), ncclUint64, ncclMax, b.comm, s),
                   "argmax all-reduce");
    cuda_check(nut::keys_to_ids(b.keys, b.B, b.ids, b.out, b.max_seq, b.ostep, s), "ids");
}

void check_gemm_error(nut_batch &b) {
    int code = 0, ar = 0;
    cuda_check(cudaMemcpyAsync(&code, b.gemm_error, sizeof code, cudaMemcpyDeviceToHost,
                               b.stream),
               "read error word");
    if (b.peers)
        cuda_check(cudaMemcpyAsync(&ar, b.ar_error, sizeof ar, cudaMemcpyDeviceToHost,
                                   b.stream),
                   "read error word");
    cuda_check(cudaStreamSynchronize(b.stream), "synchronize");
    if (ar != 0)
        raise(NUT_DEVICE_TIMEOUT, "tensor parallel: a peer all-reduce wait gave up");
    if (code != 0) {
        cudaMemsetAsync(b.gemm_error, 0, sizeof(int), b.stream);
        cudaStreamSynchronize(b.stream);
        raise(NUT_DEVICE_TIMEOUT, "device: bounded wait gave up (code " + std::to_string(code) +
                                      ")");
    }
}

/* Captures `body` (work enqueued on b.stream) as an executable graph;
 * *kernels receives how many of this library's kernels it holds. */
template <typename F> cudaGraphExec_t capture(nut_batch &b, uint64_t *kernels, F &&body) {
    cudaGraph_t graph = nullptr;
    const uint64_t before = nut::launches_so_far();
    cuda_check(cudaStreamBeginCapture(b.stream, cudaStreamCaptureModeRelaxed), "begin capture");
    try {
        body();
    } catch (...) {
        cudaStreamEndCapture(b.stream, &graph);
        if (graph)
            cudaGraphDestroy(graph);
        throw;
    }
    cuda_check(cudaStreamEndCapture(b.stream, &graph), "end capture");
    *kernels = nut::launches_so_far() - before;
    nut::uncount_launches(*kernels); /* captured, not launched */
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    cuda_check(e, "instantiate graph");
    return exec;
}

/* The prompt pass (next prompt column, forward, advance) and the decode
 * pass (advance, forward, head) as graphs. */
void ensure_graphs(nut_batch &b, int n) {
    if (b.g_prompt == nullptr || b.g_prompt_n != n) {
        if (b.g_prompt)
            cudaGraphExecDestroy(b.g_prompt);
        b.g_prompt = capture(b, &b.g_prompt_kernels, [&] {
            cuda_check(nut::prompt_column(b.prompts, b.B, n, b.pstep, b.ids, b.stream),
                       "prompt");
            forward(b);
            cuda_check(nut::advance(b.pos, b.pstep, b.stream), "advance");
        });
        b.g_prompt_n = n;
    }
    if (b.g_decode == nullptr)
        b.g_decode = capture(b, &b.g_decode_kernels, [&] {
            cuda_check(nut::advance(b.pos, b.ostep, b.stream), "advance");
            forward(b);
            head(b, false);
        });
}

nut_status create(const nut_config *config, const nut_model_view *view, uint64_t seed,
                  int device, int64_t batch, int rank, int world, const uint8_t *nccl_id,
                  nut_batch **out) {
    return guarded([&] {
        if (config == nullptr || out == nullptr || (world > 1 && nccl_id == nullptr))
            raise(NUT_INVALID_ARGUMENT, "batch: null argument");
        *out = nullptr;
        DeviceScope scope(device);
        auto b = std::make_unique<nut_batch>();
        b->device = device;
        plan_shard(*b, *config, rank, world, batch);
        alloc_state(*b);
        if (view != nullptr)
            load_view(*b, *view);
        else
            load_synthetic(*b, seed);
        if (world > 1) {
            ncclUniqueId id;
            std::memcpy(&id, nccl_id, sizeof id);
            nccl_check(nccl().comm_init_rank(&b->comm, world, id, rank), "init communicator");
        }
        cuda_check(cudaDeviceSynchronize(), "finish uploads");
        *out = b.release();
    });
}

} // namespace

extern "C" {

nut_status nut_tp_unique_id(uint8_t *id, int64_t size) {
    return guarded([&] {
        if (id == nullptr || size < int64_t(sizeof(ncclUniqueId)))
            raise(NUT_INVALID_ARGUMENT, "tensor parallel: id buffer too small");
        ncclUniqueId u;
        nccl_check(nccl().get_unique_id(&u), "unique id");
        std::memcpy(id, &u, sizeof u);
    });
}

nut_status nut_batch_create(const nut_model_view *view, int device, int64_t batch, int rank,
                            int world, const uint8_t *nccl_id, nut_batch **out) {
    if (view == nullptr) {
        nut::set_last_error("batch: null argument");
        return NUT_INVALID_ARGUMENT;
    }
    return create(&view->config, view, 0, device, batch, rank, world, nccl_id, out);
}

nut_status nut_batch_create_synthetic(const nut_config *config, uint64_t seed, int device,
                                      int64_t batch, int rank, int world,
                                      const uint8_t *nccl_id, nut_batch **out) {
    return create(config, nullptr, seed, device, batch, rank, world, nccl_id, out);
}

void nut_batch_destroy(nut_batch *b) { delete b; }

nut_status nut_tp_shard(const nut_config *config, int rank, int world, int64_t *shard) {
    return guarded([&] {
        if (config == nullptr || shard == nullptr)
            raise(NUT_INVALID_ARGUMENT, "batch: null argument");
        nut_batch b;
        plan_shard(b, *config, rank, world, 1);
        const int64_t v[8] = {int64_t(rank) * b.heads_r, b.heads_r, int64_t(rank) * b.kvh_r,
                              b.kvh_r, int64_t(rank) * b.ffn_r, b.ffn_r, b.v0, b.vocab_r};
        std::memcpy(shard, v, sizeof v);
    });
}

nut_status nut_batch_ipc_handle(nut_batch *b, uint8_t *handle, int64_t size) {
    return guarded([&] {
        if (b == nullptr || handle == nullptr || size < int64_t(sizeof(cudaIpcMemHandle_t)))
            raise(NUT_INVALID_ARGUMENT, "tensor parallel: handle buffer too small");
        DeviceScope scope(b->device);
        if (b->peer_area == nullptr) {
            const size_t bytes = peer_area_bytes(*b);
            b->peer_area = dev_alloc<uint8_t>(bytes, "alloc peer area");
            cuda_check(cudaMemset(b->peer_area, 0, bytes), "clear peer area");
            b->ar_epochs = dev_alloc<unsigned>(nut::kArChunks, "alloc epochs");
            cuda_check(cudaMemset(b->ar_epochs, 0, nut::kArChunks * 4), "clear epochs");
            b->ar_error = dev_alloc<int>(1, "alloc error word");
            cuda_check(cudaMemset(b->ar_error, 0, sizeof(int)), "clear error word");
            cuda_check(cudaDeviceSynchronize(), "clear peer area");
        }
        cudaIpcMemHandle_t h;
        cuda_check(cudaIpcGetMemHandle(&h, b->peer_area), "ipc handle");
        std::memcpy(handle, &h, sizeof h);
    });
}

nut_status nut_batch_open_peers(nut_batch *b, const uint8_t *handles, int64_t stride) {
    return guarded([&] {
        if (b == nullptr || handles == nullptr || stride < int64_t(sizeof(cudaIpcMemHandle_t)))
            raise(NUT_INVALID_ARGUMENT, "tensor parallel: invalid handles");
        if (b->peer_area == nullptr)
            raise(NUT_INVALID_ARGUMENT, "tensor parallel: export this rank's handle first");
        if (b->world > 8)
            raise(NUT_INVALID_ARGUMENT, "tensor parallel: peer all-reduce takes at most 8 ranks");
        DeviceScope scope(b->device);
        const size_t recv_bytes = size_t(2) * b->world * size_t(b->B) * b->dim * 4;
        for (int q = 0; q < b->world; q++) {
            uint8_t *base = b->peer_area;
            if (q != b->rank) {
                cudaIpcMemHandle_t h;
                std::memcpy(&h, handles + size_t(q) * size_t(stride), sizeof h);
                void *p = nullptr;
                cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                           "open peer memory");
                b->peer_open.push_back(p);
                base = static_cast<uint8_t *>(p);
            }
            b->recv_ptrs[q] = reinterpret_cast<float *>(base);
            b->flag_ptrs[q] = reinterpret_cast<unsigned *>(base + recv_bytes);
        }
        b->peers = true;
        /* graphs captured before hold NCCL calls: capture again */
        if (b->g_prompt) {
            cudaGraphExecDestroy(b->g_prompt);
            b->g_prompt = nullptr;
        }
        if (b->g_decode) {
            cudaGraphExecDestroy(b->g_decode);
            b->g_decode = nullptr;
        }
    });
}

nut_status nut_batch_set_prefill_threshold(nut_batch *b, int64_t min_tokens) {
    return guarded([&] {
        if (b == nullptr || min_tokens < 0)
            raise(NUT_INVALID_ARGUMENT, "batch: invalid argument");
        b->prefill_min = int(std::min<int64_t>(min_tokens, 1 << 30));
    });
}

nut_status nut_batch_info(const nut_batch *b, int64_t *info) {
    return guarded([&] {
        if (b == nullptr || info == nullptr)
            raise(NUT_INVALID_ARGUMENT, "batch: null argument");
        const int64_t v[8] = {b->B, b->heads_r, b->kvh_r, b->ffn_r, b->v0, b->vocab_r,
                              int64_t(b->weight_bytes), b->world};
        std::memcpy(info, v, sizeof v);
    });
}

nut_status nut_batch_stream(nut_batch *b, void **stream) {
    return guarded([&] {
        if (b == nullptr || stream == nullptr)
            raise(NUT_INVALID_ARGUMENT, "batch: null argument");
        *stream = b->stream;
    });
}

nut_status nut_batch_generate(nut_batch *b, const int32_t *prompts, int64_t n, int64_t steps,
                              int32_t *ids, float *logits, nut_generation_stats *stats) {
    return guarded([&] {
        if (b == nullptr || prompts == nullptr || (steps > 0 && ids == nullptr))
            raise(NUT_INVALID_ARGUMENT, "generation: invalid argument");
        if (n <= 0 || steps < 0 || n + steps > b->max_seq + 1 || n > b->max_seq)
            raise(NUT_INVALID_ARGUMENT, "generation: invalid prompt length");
        const int64_t V = b->cfg.vocab_size;
        for (int64_t i = 0; i < int64_t(b->B) * n; i++)
            if (prompts[i] < 0 || prompts[i] >= V)
                raise(NUT_OUT_OF_RANGE, "quantized decode: token out of range");
        DeviceScope scope(b->device);
        cudaStream_t s = b->stream;
        cuda_check(cudaMemcpyAsync(b->prompts, prompts, size_t(b->B) * n * 4,
                                   cudaMemcpyHostToDevice, s),
                   "copy prompts");
        cuda_check(cudaMemsetAsync(b->pos, 0, sizeof(int), s), "reset position");
        cuda_check(cudaMemsetAsync(b->pstep, 0, sizeof(int), s), "reset position");
        cuda_check(cudaMemsetAsync(b->ostep, 0, sizeof(int), s), "reset position");
        /* the argmax keys start at zero (a step cut short leaves them set) */
        cuda_check(cudaMemsetAsync(b->keys, 0, size_t(b->B) * sizeof(unsigned long long), s),
                   "clear keys");
        /* replayed graphs unless logits are copied out every step */
        const bool graphs = logits == nullptr && std::getenv("NUTLLM_NO_GRAPHS") == nullptr;
        if (graphs)
            ensure_graphs(*b, int(n));
        cuda_check(cudaEventRecord(b->ev[0], s), "record event");
        /* the prompt: as GEMMs over whole sequences, or one position per
         * pass (its classifier only after the last prompt token; the pass
         * before the last advances the position, so the last runs at n - 1) */
        /* (shapes the tiled prompt attention does not take keep the
         * per-pass prompt) */
        const bool gemm_prefill =
            n >= b->prefill_min && b->prefill_min > 0 &&
            nut::attention_prefill_supported(b->heads_r, b->kvh_r, b->hd, b->nqkv);
        if (gemm_prefill)
            prefill(*b, int(n));
        for (int64_t t = 0; t < n && !gemm_prefill; t++) {
            if (graphs && t + 1 < n) {
                cuda_check(cudaGraphLaunch(b->g_prompt, s), "replay prompt pass");
                nut::count_launches(unsigned(b->g_prompt_kernels));
                continue;
            }
            cuda_check(nut::prompt_column(b->prompts, b->B, int(n), b->pstep, b->ids, s),
                       "prompt");
            forward(*b);
            if (t + 1 < n)
                cuda_check(nut::advance(b->pos, b->pstep, s), "advance");
        }
        cuda_check(cudaEventRecord(b->ev[1], s), "record event");
        for (int64_t k = 0; k < steps; k++) {
            if (graphs && k > 0) {
                cuda_check(cudaGraphLaunch(b->g_decode, s), "replay decode pass");
                nut::count_launches(unsigned(b->g_decode_kernels));
                continue;
            }
            if (k > 0) {
                cuda_check(nut::advance(b->pos, b->ostep, s), "advance");
                forward(*b);
            }
            head(*b, logits != nullptr);
            if (logits != nullptr) {
                cuda_check(cudaMemcpyAsync(logits + size_t(k) * b->B * b->vocab_r, b->logits,
                                           size_t(b->B) * b->vocab_r * 4,
                                           cudaMemcpyDeviceToHost, s),
                           "copy logits");
                cuda_check(cudaMemsetAsync(b->logits, 0, size_t(b->B) * b->vocab_r * 4, s),
                           "clear logits");
            }
        }
        cuda_check(cudaEventRecord(b->ev[2], s), "record event");
        if (steps > 0) {
            std::vector<int32_t> all(size_t(b->B) * b->max_seq);
            cuda_check(cudaMemcpyAsync(all.data(), b->out, all.size() * 4,
                                       cudaMemcpyDeviceToHost, s),
                       "copy ids");
            check_gemm_error(*b);
            for (int r = 0; r < b->B; r++)
                std::memcpy(ids + size_t(r) * steps, all.data() + size_t(r) * b->max_seq,
                            size_t(steps) * 4);
        } else {
            check_gemm_error(*b);
        }
        if (stats != nullptr) {
            float pre = 0.0f, dec = 0.0f;
            cuda_check(cudaEventElapsedTime(&pre, b->ev[0], b->ev[1]), "elapsed");
            cuda_check(cudaEventElapsedTime(&dec, b->ev[1], b->ev[2]), "elapsed");
            stats->prefill_tokens = int64_t(b->B) * n;
            stats->generated_tokens = int64_t(b->B) * steps;
            stats->prefill_seconds = double(pre) * 1e-3;
            stats->decode_seconds = double(dec) * 1e-3;
        }
    });
}

static_assert(nut::kArChunks == NUT_PEER_AR_CHUNKS, "flag layout of the C ABI");

/* One peer-memory all-reduce on caller-owned buffers (see the header). */
nut_status nut_peer_all_reduce(const float *x, float *out, int64_t n, float *const *recv,
                               unsigned *const *flags, int rank, int world, unsigned *epochs,
                               int *error, int64_t limit_ns, void *stream) {
    return guarded([&] {
        if (x == nullptr || out == nullptr || recv == nullptr || flags == nullptr ||
            epochs == nullptr || error == nullptr)
            raise(NUT_INVALID_ARGUMENT, "peer all-reduce: null pointer");
        if (world < 1 || world > 8 || rank < 0 || rank >= world)
            raise(NUT_INVALID_ARGUMENT, "peer all-reduce: invalid rank or world");
        if (n <= 0 || n % 4 != 0 || n > (int64_t(1) << 28) || limit_ns <= 0)
            raise(NUT_INVALID_ARGUMENT, "peer all-reduce: invalid size or limit");
        auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
        if (!a16(x) || !a16(out))
            raise(NUT_INVALID_ARGUMENT, "peer all-reduce: buffers must be 16-byte aligned");
        for (int q = 0; q < world; q++)
            if (recv[q] == nullptr || flags[q] == nullptr || !a16(recv[q]))
                raise(NUT_INVALID_ARGUMENT, "peer all-reduce: invalid receive area");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        cuda_check(nut::peer_all_reduce(x, out, int(n), recv, flags, rank, world, epochs, error,
                                        uint64_t(limit_ns), s),
                   "peer all-reduce");
        int code = 0;
        cuda_check(cudaMemcpyAsync(&code, error, sizeof code, cudaMemcpyDeviceToHost, s),
                   "read error word");
        cuda_check(cudaStreamSynchronize(s), "peer all-reduce");
        if (code != 0) {
            cuda_check(cudaMemsetAsync(error, 0, sizeof(int), s), "clear error word");
            cuda_check(cudaStreamSynchronize(s), "clear error word");
            raise(NUT_DEVICE_TIMEOUT, "peer all-reduce: a wait for a peer's chunk gave up");
        }
    });
}

} // extern "C"
