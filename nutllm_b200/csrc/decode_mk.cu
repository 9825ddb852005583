/* The persistent token loop: every layer of every token of one generation
 * in a single cooperative launch (one CTA per SM).
 *
 * Per token i at position pos (reference decode_quantized_token,
 * src/quant_model.cpp:158-206, then the greedy head of generate_tokens_cached,
 * src/generate.cpp:197-205), for each layer l:
 *   QKV   x = rmsnorm(h) -> [q;k;v] = Wqkv x, RoPE on q and k
 *         (src/quant_model.cpp:26-37), k and v appended to the KV cache
 *   WO    GQA attention over positions 0..pos (src/quant_model.cpp:68-105),
 *         hA = h + Wo ctx
 *   GU    x = rmsnorm(hA) -> [gate;up] = Wgu x
 *   DOWN  a = silu(gate) * up, hB = hA + Wdown a
 * and, when the token's logits are needed, LMHEAD: x = rmsnorm(hB),
 * logits = W_cls x (fp32), argmax (first index of the maximum).
 *
 * Each CTA owns an even share of the row tiles of every matrix and of the
 * classifier rows, so its weights form a fixed sequence of contiguous runs
 * that its producer warp streams through the shared-memory ring without
 * ever waiting for activations: weight traffic runs ahead across phase and
 * token boundaries, limited only by the ring.  Activations cross CTAs
 * through tagged vectors: every element is written once per phase as one
 * 64-bit (value, tag) store, the tag naming the token, layer and phase, and
 * a consumer waits until every element it needs carries the expected tag.
 * That replaces grid-wide barriers with point-to-point data readiness.
 * Key and value rows of the current position travel in the tagged q|k|v
 * vector; their cache stores precede a release store of the tag, and the
 * attention's acquire loads of those tags make every earlier cache store
 * of the same owner visible.  The next token id comes from a 64-bit
 * atomicMax key per token plus a count of CTAs that finished the
 * classifier.  Every wait is bounded by limit_ns and reports into *error.
 */
#include <cmath>
#include <cstdio>

#include "decode_mk.h"
#include "kernels.h"
#include "stream.cuh"

namespace nut {
namespace {

constexpr int W = 15;            /* consumer warps (16 per CTA with the producer: 128 registers each) */
constexpr int NT = W * 32;       /* consumer threads */
constexpr int THREADS = NT + 32; /* + the producer warp */
constexpr int kBar = 1;          /* named barrier of the consumer warps */

__device__ __forceinline__ uint64_t ld_relaxed(const Tagged *p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ld_acquire(const Tagged *p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed(Tagged *p, float v, uint32_t tag) {
    const uint64_t x = (uint64_t(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;\n" ::"l"(p), "l"(x) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void cbar() { named_barrier(kBar, NT); }

/* 4-byte asynchronous global -> shared copy (no register round trip). */
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;\n" ::: "memory");
}

/* Phases per layer: 0 QKV, 1 ATT, 2 WO, 3 GU, 4 DOWN. */
__device__ __forceinline__ uint32_t tag_of(const MkParams &p, int i, int l, int phase) {
    return 1u + uint32_t((i * p.layers + l) * 5 + phase);
}

/* Row-tile (or row) range of this CTA in an even split of `total`
 * (total * gridDim.x < 2^31 for every supported shape; 32-bit arithmetic
 * avoids the emulated 64-bit division). */
__device__ __forceinline__ void share(int total, int &a, int &b) {
    const unsigned t = unsigned(total), c = gridDim.x, i = blockIdx.x;
    a = int(t * i / c);
    b = int(t * (i + 1) / c);
}

struct Shared {
    Ring ring;
    float *xvec;       /* [kmax] staged activations */
    int8_t *dig;       /* union region: digits ... */
    float *fac;
    float *uni;        /* ... or attention scratch */
    float *red;        /* [2][kRowBatch][W][16] */
    float *wsum;       /* [W] */
    unsigned long long *bestk; /* [W] */
    int *flag;         /* [0] fatal, [1] token */
    float *res;        /* [kResRows] residual inputs of this CTA's rows */
};

/* Optional phase trace (thread 0 of each CTA): one record of 8 words per
 * phase occurrence: phase id, the global timer at entry (1), and SM clock
 * stamps at entry (6), inputs staged (2), activation ready (3), digits
 * ready (4), weights consumed (5) and exit (7). */
struct Trace {
    unsigned long long *rec = nullptr;
    __device__ __forceinline__ void open(const MkParams &p, int occ, int id) {
        waited = 0;
        rec = p.trace != nullptr && occ < p.trace_stride
                  ? p.trace + (size_t(blockIdx.x) * p.trace_stride + occ) * 8
                  : nullptr;
        if (rec != nullptr && threadIdx.x == 0) {
            rec[0] = unsigned(id);
            rec[1] = global_ns();
            rec[6] = clock64();
        }
    }
    /* slots 2-5 and 7: SM clock (cycles) */
    __device__ __forceinline__ void mark(int slot) const {
        if (rec != nullptr && threadIdx.x == 0)
            rec[slot] = clock64();
    }
    /* slot 3 of consume phases: cycles warp 0 waited for weight stages */
    long long waited = 0;
    __device__ __forceinline__ long long *wait_acc() {
        return rec != nullptr && threadIdx.x == 0 ? &waited : nullptr;
    }
    __device__ __forceinline__ void put_wait() const {
        if (rec != nullptr && threadIdx.x == 0)
            rec[3] = (unsigned long long)waited;
    }
};

template <int STAGES>
__device__ Shared carve(uint8_t *base, const MkParams &p) {
    Shared s;
    size_t off = 0;
    uint8_t *data = base;
    off += size_t(STAGES) * kStageBytes;
    uint16_t *scales = reinterpret_cast<uint16_t *>(base + off);
    off += size_t(STAGES) * kStageScaleBytes;
    const int kmax = p.dim > p.ffn ? p.dim : p.ffn;
    s.xvec = reinterpret_cast<float *>(base + off);
    off += size_t(kmax) * 4;
    off = (off + 15) & ~size_t(15);
    s.uni = reinterpret_cast<float *>(base + off);
    s.dig = reinterpret_cast<int8_t *>(base + off);
    const int nbmax = p.nb_dim > p.nb_ffn ? p.nb_dim : p.nb_ffn;
    s.fac = reinterpret_cast<float *>(base + off + size_t(nbmax) * 128);
    off += size_t(p.union_floats) * 4;
    off = (off + 15) & ~size_t(15);
    auto align16 = [](size_t o) { return (o + 15) & ~size_t(15); };
    s.red = reinterpret_cast<float *>(base + off);
    off = align16(off + 2 * kRowBatch * W * 16 * 4);
    s.wsum = reinterpret_cast<float *>(base + off);
    off = align16(off + W * 4);
    s.bestk = reinterpret_cast<unsigned long long *>(base + off);
    off = align16(off + W * 8);
    s.flag = reinterpret_cast<int *>(base + off);
    off = align16(off + 16);
    s.res = reinterpret_cast<float *>(base + off);
    off = align16(off + 64 * 4);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + off);
    s.ring = Ring{data, scales, bars, bars + STAGES, STAGES, p.limit_ns, p.error, s.flag};
    return s;
}

/* Deterministic sum over the consumer threads. */
__device__ __forceinline__ float csum(const Shared &s, float v) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0)
        s.wsum[warp] = v;
    cbar();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < W; w++)
        t += s.wsum[w];
    cbar();
    return t;
}

/* Collective: true when no consumer has hit a fatal condition. */
__device__ __forceinline__ bool healthy(const Shared &s) {
    cbar();
    return *reinterpret_cast<volatile int *>(s.flag) == 0;
}

__device__ __forceinline__ void fatal(const Shared &s, const MkParams &p, int code) {
    *reinterpret_cast<volatile int *>(s.flag) = 1;
    report(p.error, code);
}

/* Waits for one tagged element. */
template <bool ACQ>
__device__ __forceinline__ bool wait_tag(const Tagged *src, uint32_t tag,
                                         uint64_t limit, float &v) {
    uint64_t x = ACQ ? ld_acquire(src) : ld_relaxed(src);
    if (uint32_t(x >> 32) != tag) {
        const uint64_t t0 = global_ns();
        do {
            __nanosleep(64);
            x = ACQ ? ld_acquire(src) : ld_relaxed(src);
            if (uint32_t(x >> 32) == tag)
                break;
            if (global_ns() - t0 > limit)
                return false;
        } while (true);
    }
    v = __uint_as_float(uint32_t(x));
    return true;
}

constexpr int kPollBatch = 8; /* element loads in flight per thread */

/* Loads up to kPollBatch tagged elements k0, k0 + NT, ... (< n) of src
 * into v[] with all loads issued before any tag is checked; retries (with
 * a short sleep) until every tag matches.  False on timeout. */
template <bool ACQ>
__device__ __forceinline__ bool wait_batch(const Tagged *src, int n, int k0,
                                           uint32_t tag, uint64_t limit,
                                           float (&v)[kPollBatch]) {
    uint64_t x[kPollBatch];
    uint64_t t0 = 0;
    for (bool first = true;; first = false) {
#pragma unroll
        for (int j = 0; j < kPollBatch; j++) {
            const int k = k0 + j * NT;
            x[j] = k < n ? (ACQ ? ld_acquire(src + k) : ld_relaxed(src + k))
                         : (uint64_t(tag) << 32);
        }
        bool ready = true;
#pragma unroll
        for (int j = 0; j < kPollBatch; j++)
            ready = ready && uint32_t(x[j] >> 32) == tag;
        if (ready)
            break;
        const uint64_t now = global_ns();
        if (first)
            t0 = now;
        else if (now - t0 > limit)
            return false;
        __nanosleep(128);
    }
#pragma unroll
    for (int j = 0; j < kPollBatch; j++)
        v[j] = __uint_as_float(uint32_t(x[j]));
    return true;
}

/* Collective: stages n tagged elements into dst; thread t handles elements
 * t, t + NT, ... */
template <bool ACQ>
__device__ bool poll(const Shared &s, const MkParams &p, const Tagged *src, int n,
                     uint32_t tag, float *dst) {
    for (int k0 = threadIdx.x; k0 < n; k0 += kPollBatch * NT) {
        float v[kPollBatch];
        /* acquire = relaxed loads of every tag, then one fence */
        if (!wait_batch<false>(src, n, k0, tag, p.limit_ns, v)) {
            fatal(s, p, kErrTimeoutInput);
            break;
        }
#pragma unroll
        for (int j = 0; j < kPollBatch; j++)
            if (k0 + j * NT < n)
                dst[k0 + j * NT] = v[j];
    }
    if (ACQ)
        __threadfence();
    return healthy(s);
}

/* Norm weights of this thread's elements (k = tid + j NT), loaded before
 * the inputs are polled so their latency overlaps the wait. */
struct NormW {
    float w[kPollBatch];
    __device__ __forceinline__ void load(const float *src, int n) {
#pragma unroll
        for (int j = 0; j < kPollBatch; j++) {
            const int k = threadIdx.x + j * NT;
            w[j] = k < n ? __ldg(src + k) : 0.0f;
        }
    }
};

/* In-place rmsnorm over xvec[0..n) staged by poll (same thread mapping,
 * n <= kPollBatch * NT): x * (1 / sqrt(mean(x^2) + eps)) * w
 * (src/ops.cpp:111-134). */
__device__ void rmsnorm_staged(const Shared &s, int n, const NormW &nw) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kPollBatch; j++) {
        const int k = threadIdx.x + j * NT;
        if (k < n)
            ss = fmaf(s.xvec[k], s.xvec[k], ss);
    }
    const float total = csum(s, ss);
    const float scale = 1.0f / sqrtf(total / float(n) + kEps);
#pragma unroll
    for (int j = 0; j < kPollBatch; j++) {
        const int k = threadIdx.x + j * NT;
        if (k < n)
            s.xvec[k] = s.xvec[k] * scale * nw.w[j];
    }
    cbar();
}

template <int TYPE>
__device__ __forceinline__ void digits(const Shared &s, int K, int nb) {
    make_digits(s.xvec, K, nb, threadIdx.x >> 5, W, s.dig, s.fac,
                TYPE == 1 ? 1.0f / 16.0f : 1.0f);
    cbar();
}

/* Interleaved-pair RoPE of the pair (lane, lane ^ 1) with unfused products,
 * the rounding of src/quant_model.cpp:34-35. */
__device__ __forceinline__ float rope(float y, int lane, float c, float sn) {
    const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
    return (lane & 1) ? __fadd_rn(__fmul_rn(partner, sn), __fmul_rn(y, c))
                      : __fsub_rn(__fmul_rn(y, c), __fmul_rn(partner, sn));
}

/* ---- warp-sliced phase prologue ---------------------------------------

   Consumer warp w multiplies block pairs p = w, w + W, ... of every row
   tile, i.e. always the same K slice.  It therefore stages, normalises and
   digitises only its own slice, in registers, and starts its tensor-core
   work without waiting for the rest of the CTA.  For the rmsnorm phases the
   digitised vector is u = h * norm_weight; the scale 1/sqrt(mean(h^2) +
   eps) is a scalar that factors out of the product (W (s u) = s (W u)) and
   is applied to each row in the epilogue, from per-warp partial sums that
   the first row-tile barrier publishes. */

constexpr int kSliceBlocks = 4; /* blocks staged per round (per lane: one element each) */

/* Element of the warp's k-th owned block: block index, or -1 past the end. */
__device__ __forceinline__ int slice_block(int w, int nb, int k) {
    const int p = w + (k >> 1) * W;
    return 2 * p < nb ? 2 * p + (k & 1) : -1;
}

/* Stages the warp's slice of an input vector of K elements (tagged, or a
 * plain fp32 row when `plain` is set), multiplies it by `norm` (if any),
 * writes its digits and block factors and returns the lane's sum of
 * squares of the raw inputs.  False on timeout. */
template <int TYPE>
__device__ bool warp_slice(const Shared &s, const MkParams &p, const Tagged *src,
                           const float *plain, int K, int nb, uint32_t tag,
                           const float *norm, float &ss) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float a_unit_inv = TYPE == 1 ? 1.0f / 16.0f : 1.0f;
    ss = 0.0f;
    for (int k0 = 0;; k0 += kSliceBlocks) {
        if (slice_block(w, nb, k0) < 0)
            break;
        float nw[kSliceBlocks];
        uint64_t x[kSliceBlocks];
#pragma unroll
        for (int k = 0; k < kSliceBlocks; k++) {
            const int b = slice_block(w, nb, k0 + k), e = b * 32 + lane;
            const bool in = b >= 0 && e < K;
            nw[k] = norm != nullptr && in ? __ldg(norm + e) : 1.0f;
            if (plain != nullptr)
                x[k] = (uint64_t(tag) << 32) | __float_as_uint(in ? plain[e] : 0.0f);
            else
                x[k] = in ? ld_relaxed(src + e) : (uint64_t(tag) << 32);
        }
        if (plain == nullptr) {
            uint64_t t0 = 0;
            for (bool first = true;; first = false) {
                bool ready = true;
#pragma unroll
                for (int k = 0; k < kSliceBlocks; k++)
                    ready = ready && uint32_t(x[k] >> 32) == tag;
                if (__all_sync(0xffffffffu, ready))
                    break;
                const uint64_t now = global_ns();
                if (first)
                    t0 = now;
                else if (now - t0 > p.limit_ns) {
                    fatal(s, p, kErrTimeoutInput);
                    return false;
                }
                __nanosleep(128);
#pragma unroll
                for (int k = 0; k < kSliceBlocks; k++) {
                    const int b = slice_block(w, nb, k0 + k), e = b * 32 + lane;
                    if (b >= 0 && e < K && uint32_t(x[k] >> 32) != tag)
                        x[k] = ld_relaxed(src + e);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kSliceBlocks; k++) {
            const int b = slice_block(w, nb, k0 + k);
            if (b < 0)
                break;
            const float v = __uint_as_float(uint32_t(x[k]));
            ss = fmaf(v, v, ss);
            const float u = v * nw[k];
            s.xvec[b * 32 + lane] = u;
            digit_block(s.xvec, nb * 32, b, s.dig, s.fac, a_unit_inv);
        }
    }
    return true;
}

/* Publishes the warp's sum of squares for the epilogue's norm scale. */
__device__ __forceinline__ void slice_ss(const Shared &s, float ss) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0)
        s.wsum[threadIdx.x >> 5] = ss;
    __syncwarp();
}

/* rmsnorm scale from the published partial sums (read after a barrier). */
__device__ __forceinline__ float norm_scale(const Shared &s, int n) {
    float v[W];
#pragma unroll
    for (int k = 0; k < W; k++)
        v[k] = s.wsum[k];
#pragma unroll
    for (int step = 1; step < W; step *= 2)
#pragma unroll
        for (int k = 0; k + step < W; k += 2 * step)
            v[k] += v[k + step];
    return 1.0f / sqrtf(v[0] / float(n) + kEps);
}

/* ---------------------------------------------------------------- phases */

template <int TYPE, int STAGES>
__device__ bool phase_qkv(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                          RowReduce &rr, int i, int l, int token, int pos) {
    int a, b;
    share(p.rt_qkv, a, b);
    if (a == b)
        return true;
    float ss;
    if (!warp_slice<TYPE>(s, p, p.hB, l == 0 ? p.emb + size_t(token) * p.dim : nullptr, p.dim,
                          p.nb_dim, l == 0 ? 0u : tag_of(p, i, l - 1, 4),
                          p.attn_norm + size_t(l) * p.dim, ss))
        ss = 0.0f;
    slice_ss(s, ss);
    tr.mark(2);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const TileRun run{L.qkv + size_t(a) * p.nb_dim * TB, L.qkv_s + size_t(a) * p.nb_dim * 16,
                      (b - a) * p.nb_dim, p.nb_dim};
    const uint32_t tag = tag_of(p, i, l, 0);
    const int lane = threadIdx.x & 31, half = p.hd / 2;
    const float *cs = p.rope_cos + size_t(pos) * half;
    const float *sn = p.rope_sin + size_t(pos) * half;
    /* The cache rows of this token are read only by later tokens: the
     * fence ahead of each token's key/value tags orders the rows written
     * by the same lane one token earlier, and the readers acquire those
     * tags (load, then fence) before fetching history. */
    auto epi = [&](int rt, float y) {
        y *= norm_scale(s, p.dim);
        const int row0 = (a + rt) * 16, row = row0 + (lane & 15);
        if (row0 < p.dim) {                       /* query */
            const int j = (row % p.hd) >> 1;
            const float out = rope(y, lane, cs[j], sn[j]);
            if (lane < 16)
                st_relaxed(p.qkv + row, out, tag);
        } else if (row0 < p.dim + p.kvd) {        /* key */
            const int kr = row - p.dim, h = kr / p.hd, d = kr % p.hd;
            const float out = rope(y, lane, cs[d >> 1], sn[d >> 1]);
            if (lane < 16) {
                __threadfence();
                st_relaxed(p.qkv + row, out, tag);
                p.kcache[((size_t(l) * p.kv_heads + h) * p.max_seq + pos) * p.hd + d] = out;
            }
        } else if (lane < 16) {                   /* value */
            const int vr = row - p.dim - p.kvd, h = vr / p.hd, d = vr % p.hd;
            __threadfence();
            st_relaxed(p.qkv + row, y, tag);
            p.vcache[((size_t(l) * p.kv_heads + h) * p.max_seq + pos) * p.hd + d] = y;
        }
    };
    const bool ok = consume_run<TYPE, W, STAGES>(s.ring, run, cur, s.dig, s.fac, rr,
                                                 threadIdx.x >> 5, kBar, epi,
                                                 tr.wait_acc());
    tr.mark(5);
    tr.put_wait();
    return healthy(s) && ok;
}

/* Query heads owned by this CTA: head h belongs to CTA floor(h C / H),
 * i.e. this CTA owns h in [ceil(c H / C), ceil((c + 1) H / C)). */
__device__ __forceinline__ void owned_heads(int heads, int &h0, int &h1) {
    const unsigned H = unsigned(heads), C = gridDim.x, c = blockIdx.x;
    h0 = int((c * H + C - 1) / C);
    h1 = int(((c + 1) * H + C - 1) / C);
}

/* Per-head attention scratch inside the union region. */
struct HeadScratch {
    float *q;        /* [hd] */
    float *Kt, *Vt;  /* [CH][hd + 1] (padded rows: conflict-free) */
    float *w;        /* [CH] scores, then exp weights */
    float *part;     /* [NT] partial context sums */
    float *stat;     /* [2]: running max, running sum */
    int CH;
    __device__ HeadScratch(const Shared &s, const MkParams &p) {
        const int hd = p.hd, ld = hd + 1;
        q = s.uni;
        stat = q + hd;
        part = stat + 2;
        w = part + NT;
        const int used = hd + 2 + NT;
        CH = (p.union_floats - used) / (2 * ld + 1);
        if (CH > NT)
            CH = NT;
        Kt = w + CH;
        Vt = Kt + CH * ld;
    }
};

/* Asynchronous copies of cached keys and values of kv head g, positions
 * [p0, p0 + n) other than `pos`, into the tiles. */
__device__ __forceinline__ void head_fetch(const HeadScratch &t, const MkParams &p, int l,
                                           int g, int p0, int n, int pos) {
    const int hd = p.hd, ld = hd + 1;
    const size_t base = (size_t(l) * p.kv_heads + g) * size_t(p.max_seq) * hd;
    for (int idx = threadIdx.x; idx < n * hd; idx += NT) {
        const int j = idx / hd, d = idx - j * hd, q = p0 + j;
        if (q == pos)
            continue;
        const size_t off = base + size_t(q) * hd + d;
        cp_async4(t.Kt + j * ld + d, p.kcache + off);
        cp_async4(t.Vt + j * ld + d, p.vcache + off);
    }
}

/* Block-wide max / sum over the consumer threads (all threads get it). */
__device__ __forceinline__ float cmax(const Shared &s, float v) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0)
        s.wsum[threadIdx.x >> 5] = v;
    cbar();
    float t = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; w++)
        t = fmaxf(t, s.wsum[w]);
    cbar();
    return t;
}

/* ATT: the heads this CTA owns, each over positions 0..pos in chunks
 * (attention_step, src/quant_model.cpp:68-105: scores q.k / sqrt(hd),
 * exp(score - max), weights / total, context); the context of head h is
 * published as tagged elements ctx[h hd .. h hd + hd). */
__device__ bool phase_att(const Shared &s, const MkParams &p, Trace &tr, int i, int l,
                          int pos) {
    const int H = p.heads, hd = p.hd, ld = hd + 1, G = p.heads / p.kv_heads;
    const uint32_t tag_in = tag_of(p, i, l, 0), tag = tag_of(p, i, l, 1);
    const float scale = 1.0f / sqrtf(float(hd));
    const HeadScratch t(s, p);
    const int slices = NT / hd; /* position slices in the context sum */
    int h_first, h_last;
    owned_heads(H, h_first, h_last);
    for (int h = h_first; h < h_last; h++) {
        const int g = h / G;
        /* history does not depend on this token: fetch it first */
        head_fetch(t, p, l, g, 0, min(t.CH, pos + 1), pos);
        /* q of head h and the current k, v of kv head g */
        bool ok = true;
        if (threadIdx.x < 3 * hd) {
            const int part = threadIdx.x / hd, d = threadIdx.x - part * hd;
            const int row = part == 0 ? h * hd + d
                                      : p.dim + (part - 1) * p.kvd + g * hd + d;
            float v;
            ok = wait_tag<false>(p.qkv + row, tag_in, p.limit_ns, v);
            if (ok) {
                if (part == 0)
                    t.q[d] = v;
                else if (pos < t.CH)
                    (part == 1 ? t.Kt : t.Vt)[pos * ld + d] = v;
                else
                    t.part[d + (part - 1) * hd] = v; /* kept for its chunk */
            } else {
                fatal(s, p, kErrTimeoutInput);
            }
        }
        __threadfence(); /* acquire: the tags order the older cache rows */
        if (!healthy(s)) {
            cp_async_wait_all();
            return false;
        }
        if (threadIdx.x == 0)
            tr.mark(2);
        float m = -INFINITY, total = 0.0f, acc = 0.0f; /* acc: ctx[d] of slice */
        const int d_own = threadIdx.x % hd, sl = threadIdx.x / hd;
        float kcur = 0.0f, vcur = 0.0f;
        if (pos >= t.CH && threadIdx.x < hd) {
            kcur = t.part[threadIdx.x];
            vcur = t.part[hd + threadIdx.x];
        }
        cbar();
        for (int p0 = 0; p0 <= pos; p0 += t.CH) {
            const int n = min(t.CH, pos + 1 - p0);
            if (p0 > 0) {
                head_fetch(t, p, l, g, p0, n, pos);
                if (pos >= p0 && pos < p0 + n && threadIdx.x < hd) {
                    t.Kt[(pos - p0) * ld + threadIdx.x] = kcur;
                    t.Vt[(pos - p0) * ld + threadIdx.x] = vcur;
                }
            }
            cp_async_wait_all();
            cbar();
            float sc = -INFINITY;
            if (threadIdx.x < n) {
                const float *kj = t.Kt + threadIdx.x * ld;
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                int d = 0;
                for (; d + 4 <= hd; d += 4) {
                    a0 = fmaf(t.q[d], kj[d], a0);
                    a1 = fmaf(t.q[d + 1], kj[d + 1], a1);
                    a2 = fmaf(t.q[d + 2], kj[d + 2], a2);
                    a3 = fmaf(t.q[d + 3], kj[d + 3], a3);
                }
                for (; d < hd; d++)
                    a0 = fmaf(t.q[d], kj[d], a0);
                sc = ((a0 + a1) + (a2 + a3)) * scale;
            }
            const float m_new = fmaxf(m, cmax(s, sc));
            const float e = threadIdx.x < n ? expf(sc - m_new) : 0.0f;
            if (threadIdx.x < n)
                t.w[threadIdx.x] = e;
            const float alpha = expf(m - m_new);
            total = total * alpha + csum(s, e); /* csum's barriers publish w */
            m = m_new;
            acc *= alpha;
            if (sl < slices)
                for (int j = sl; j < n; j += slices)
                    acc = fmaf(t.w[j], t.Vt[j * ld + d_own], acc);
            cbar();
        }
        tr.mark(3);
        if (sl < slices)
            t.part[threadIdx.x] = acc;
        cbar();
        tr.mark(4);
        if (threadIdx.x < hd) {
            float c = 0.0f;
            for (int k = 0; k < slices; k++)
                c += t.part[k * hd + threadIdx.x];
            st_relaxed(p.ctx + h * hd + threadIdx.x, c / total, tag);
        }
        cbar();
        tr.mark(5);
    }
    return true;
}

/* Residual inputs of this CTA's rows, loaded without waiting before the
 * phase input is polled (their tags are normally complete by then) and
 * parked in `res` (at most kResRows rows; later rows are read in the
 * epilogue). */
constexpr int kResRows = 64;

__device__ __forceinline__ uint64_t res_issue(const Tagged *src, int row0, int nrows) {
    return threadIdx.x < nrows && threadIdx.x < kResRows
               ? ld_relaxed(src + row0 + threadIdx.x)
               : 0ull;
}

__device__ __forceinline__ void res_park(const Shared &s, const MkParams &p,
                                         const Tagged *src, int row0, int nrows,
                                         uint32_t tag, uint64_t x) {
    if (threadIdx.x < nrows && threadIdx.x < kResRows) {
        float v = __uint_as_float(uint32_t(x));
        if (uint32_t(x >> 32) != tag &&
            !wait_tag<false>(src + row0 + threadIdx.x, tag, p.limit_ns, v))
            fatal(s, p, kErrTimeoutInput);
        s.res[threadIdx.x] = v;
    }
}

template <int TYPE, int STAGES>
__device__ bool phase_wo(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                         RowReduce &rr, int i, int l, int token) {
    int a, b;
    share(p.rt_wo, a, b);
    if (a == b)
        return true;
    const int row0 = a * 16, nrows = (b - a) * 16;
    const uint32_t tag = tag_of(p, i, l, 2), tag_in = l > 0 ? tag_of(p, i, l - 1, 4) : 0;
    const uint64_t pre = l > 0 ? res_issue(p.hB, row0, nrows) : 0ull;
    if (l == 0 && threadIdx.x < nrows && threadIdx.x < kResRows)
        s.res[threadIdx.x] = p.emb[size_t(token) * p.dim + row0 + threadIdx.x];
    float ss;
    warp_slice<TYPE>(s, p, p.ctx, nullptr, p.dim, p.nb_dim, tag_of(p, i, l, 1), nullptr, ss);
    if (l > 0)
        res_park(s, p, p.hB, row0, nrows, tag_in, pre);
    tr.mark(2);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const TileRun run{L.wo + size_t(a) * p.nb_dim * TB, L.wo_s + size_t(a) * p.nb_dim * 16,
                      (b - a) * p.nb_dim, p.nb_dim};
    const int lane = threadIdx.x & 31;
    auto epi = [&](int rt, float y) {
        const int k = rt * 16 + lane, row = row0 + k;
        if (lane >= 16)
            return;
        float h;
        if (k < kResRows)
            h = s.res[k];
        else if (l == 0)
            h = p.emb[size_t(token) * p.dim + row];
        else if (!wait_tag<false>(p.hB + row, tag_in, p.limit_ns, h)) {
            fatal(s, p, kErrTimeoutInput);
            return;
        }
        st_relaxed(p.hA + row, h + y, tag);
    };
    const bool ok = consume_run<TYPE, W, STAGES>(s.ring, run, cur, s.dig, s.fac, rr,
                                                 threadIdx.x >> 5, kBar, epi,
                                                 tr.wait_acc());
    tr.mark(5);
    tr.put_wait();
    return healthy(s) && ok;
}

template <int TYPE, int STAGES>
__device__ bool phase_gu(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                         RowReduce &rr, int i, int l) {
    int a, b;
    share(p.rt_gu, a, b);
    if (a == b)
        return true;
    float ss;
    if (!warp_slice<TYPE>(s, p, p.hA, nullptr, p.dim, p.nb_dim, tag_of(p, i, l, 2),
                          p.ffn_norm + size_t(l) * p.dim, ss))
        ss = 0.0f;
    slice_ss(s, ss);
    tr.mark(2);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const TileRun run{L.gu + size_t(a) * p.nb_dim * TB, L.gu_s + size_t(a) * p.nb_dim * 16,
                      (b - a) * p.nb_dim, p.nb_dim};
    const uint32_t tag = tag_of(p, i, l, 3);
    const int lane = threadIdx.x & 31;
    /* tile rt: lanes 0-7 gate rows, lanes 8-15 up rows of units 8 R .. 8 R + 7;
     * a = silu(gate) * up (src/quant_model.cpp:197-198) */
    auto epi = [&](int rt, float y) {
        y *= norm_scale(s, p.dim);
        const float up = __shfl_down_sync(0xffffffffu, y, 8);
        if (lane < 8)
            st_relaxed(p.act + (a + rt) * 8 + lane, y / (1.0f + expf(-y)) * up, tag);
    };
    const bool ok = consume_run<TYPE, W, STAGES>(s.ring, run, cur, s.dig, s.fac, rr,
                                                 threadIdx.x >> 5, kBar, epi,
                                                 tr.wait_acc());
    tr.mark(5);
    tr.put_wait();
    return healthy(s) && ok;
}

template <int TYPE, int STAGES>
__device__ bool phase_down(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                           RowReduce &rr, int i, int l) {
    int a, b;
    share(p.rt_down, a, b);
    if (a == b)
        return true;
    const int row0 = a * 16, nrows = (b - a) * 16;
    const uint32_t tag = tag_of(p, i, l, 4), tag_in = tag_of(p, i, l, 2);
    const uint64_t pre = res_issue(p.hA, row0, nrows);
    float ss;
    warp_slice<TYPE>(s, p, p.act, nullptr, p.ffn, p.nb_ffn, tag_of(p, i, l, 3), nullptr, ss);
    res_park(s, p, p.hA, row0, nrows, tag_in, pre);
    tr.mark(2);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const TileRun run{L.down + size_t(a) * p.nb_ffn * TB,
                      L.down_s + size_t(a) * p.nb_ffn * 16, (b - a) * p.nb_ffn, p.nb_ffn};
    const int lane = threadIdx.x & 31;
    auto epi = [&](int rt, float y) {
        const int k = rt * 16 + lane, row = row0 + k;
        if (lane >= 16)
            return;
        float h;
        if (k < kResRows)
            h = s.res[k];
        else if (!wait_tag<false>(p.hA + row, tag_in, p.limit_ns, h)) {
            fatal(s, p, kErrTimeoutInput);
            return;
        }
        st_relaxed(p.hB + row, h + y, tag);
    };
    const bool ok = consume_run<TYPE, W, STAGES>(s.ring, run, cur, s.dig, s.fac, rr,
                                                 threadIdx.x >> 5, kBar, epi,
                                                 tr.wait_acc());
    tr.mark(5);
    tr.put_wait();
    return healthy(s) && ok;
}

__device__ __forceinline__ int lm_rows_per_chunk(const MkParams &p) {
    return kStageBytes / (p.dim * 4);
}

template <int STAGES>
__device__ bool phase_lmhead(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                             int i) {
    int a, b;
    share(p.vocab, a, b);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long best = 0ull;
    if (a < b) {
        NormW nw;
        nw.load(p.final_norm, p.dim);
        if (!poll<false>(s, p, p.hB, p.dim, tag_of(p, i, p.layers - 1, 4), s.xvec))
            return false;
        if (i == p.n_prompt - 1 && blockIdx.x == 0 && threadIdx.x == 0)
            p.stamps[1] = global_ns(); /* every layer of the prompt is done */
        tr.mark(2);
        rmsnorm_staged(s, p.dim, nw);
        const int CR = lm_rows_per_chunk(p), d4 = p.dim / 4;
        const float4 *x4 = reinterpret_cast<const float4 *>(s.xvec);
        float *out = p.logits ? p.logits + size_t(i - p.logits_from) * p.vocab : nullptr;
        for (int r0 = a; r0 < b; r0 += CR) {
            const int nr = min(CR, b - r0);
            if (*reinterpret_cast<volatile int *>(s.flag) != 0)
                break;
            if (!mbar_wait(&s.ring.full[cur.stage], cur.parity, p.limit_ns)) {
                fatal(s, p, kErrTimeoutFull);
                break;
            }
            const float4 *rows = reinterpret_cast<const float4 *>(
                s.ring.data + size_t(cur.stage) * kStageBytes);
            for (int j = 0; j < nr; j++) {
                if ((r0 - a + j) % W != warp)
                    continue;
                const float4 *w4 = rows + size_t(j) * d4;
                float acc = 0.0f;
                for (int g = lane; g < d4; g += 32) {
                    const float4 w = w4[g], x = x4[g];
                    acc = fmaf(w.x, x.x, acc);
                    acc = fmaf(w.y, x.y, acc);
                    acc = fmaf(w.z, x.z, acc);
                    acc = fmaf(w.w, x.w, acc);
                }
                acc = warp_sum(acc);
                if (lane == 0) {
                    if (out)
                        out[r0 + j] = acc;
                    const unsigned long long k = argmax_key(acc, uint32_t(r0 + j));
                    best = k > best ? k : best;
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.ring.empty[cur.stage]);
            cur.template next<STAGES>();
        }
    }
    if (lane == 0)
        s.bestk[warp] = best;
    if (!healthy(s))
        return false;
    if (threadIdx.x == 0) {
        unsigned long long m = 0ull;
        for (int w = 0; w < W; w++)
            m = s.bestk[w] > m ? s.bestk[w] : m;
        if (m != 0ull)
            atomicMax(p.keys + i, m);
        __threadfence();
        atomicAdd(p.done + i, 1u);
    }
    return true;
}

/* Token id of step i >= n_prompt: the argmax of step i - 1, once every CTA
 * has contributed to it. */
__device__ bool next_token(const Shared &s, const MkParams &p, int i, int &token) {
    if (threadIdx.x == 0) {
        const unsigned want = gridDim.x;
        const uint64_t t0 = global_ns();
        bool ok = true;
        while (ld_acquire_u32(p.done + (i - 1)) < want) {
            if (global_ns() - t0 > p.limit_ns) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
        if (ok) {
            const unsigned long long k =
                *reinterpret_cast<volatile unsigned long long *>(p.keys + (i - 1));
            const uint32_t t = argmax_index(k);
            s.flag[1] = t < uint32_t(p.vocab) ? int(t) : 0;
        } else {
            fatal(s, p, kErrTimeoutInput);
        }
    }
    if (!healthy(s))
        return false;
    token = s.flag[1];
    return true;
}

__device__ __forceinline__ bool wants_logits(const MkParams &p, int i) {
    return i >= p.logits_from && i <= p.logits_to;
}

template <int TYPE, int STAGES>
__device__ void producer(const Shared &s, const MkParams &p) {
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    Cursor cur;
    for (int i = 0; i < p.n_tokens; i++) {
        for (int l = 0; l < p.layers; l++) {
            const MkLayerPtrs &L = p.layer[l];
            int a, b;
            share(p.rt_qkv, a, b);
            if (a < b &&
                !produce_run_c<TYPE, STAGES>(s.ring,
                    TileRun{L.qkv + size_t(a) * p.nb_dim * TB, L.qkv_s + size_t(a) * p.nb_dim * 16,
                            (b - a) * p.nb_dim, p.nb_dim}, cur))
                return;
            share(p.rt_wo, a, b);
            if (a < b &&
                !produce_run_c<TYPE, STAGES>(s.ring,
                    TileRun{L.wo + size_t(a) * p.nb_dim * TB, L.wo_s + size_t(a) * p.nb_dim * 16,
                            (b - a) * p.nb_dim, p.nb_dim}, cur))
                return;
            share(p.rt_gu, a, b);
            if (a < b &&
                !produce_run_c<TYPE, STAGES>(s.ring,
                    TileRun{L.gu + size_t(a) * p.nb_dim * TB, L.gu_s + size_t(a) * p.nb_dim * 16,
                            (b - a) * p.nb_dim, p.nb_dim}, cur))
                return;
            share(p.rt_down, a, b);
            if (a < b &&
                !produce_run_c<TYPE, STAGES>(s.ring,
                    TileRun{L.down + size_t(a) * p.nb_ffn * TB,
                            L.down_s + size_t(a) * p.nb_ffn * 16, (b - a) * p.nb_ffn, p.nb_ffn},
                    cur))
                return;
        }
        if (wants_logits(p, i)) {
            int a, b;
            share(p.vocab, a, b);
            const int CR = lm_rows_per_chunk(p);
            for (int r0 = a; r0 < b; r0 += CR) {
                const int nr = min(CR, b - r0);
                if (!mbar_wait(&s.ring.empty[cur.stage], cur.parity ^ 1u, p.limit_ns)) {
                    report(p.error, kErrTimeoutEmpty);
                    return;
                }
                const uint32_t bytes = uint32_t(nr) * uint32_t(p.dim) * 4u;
                mbar_expect_tx(&s.ring.full[cur.stage], bytes);
                bulk_g2s(s.ring.data + size_t(cur.stage) * kStageBytes,
                         p.lm_head + size_t(r0) * p.dim, bytes, &s.ring.full[cur.stage]);
                cur.template next<STAGES>();
            }
        }
    }
}

template <int TYPE, int STAGES>
__global__ void __launch_bounds__(THREADS, 1) decode_mk_kernel(const MkParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    Shared s = carve<STAGES>(smem, p);
    if (threadIdx.x == 0) {
        for (int k = 0; k < STAGES; k++) {
            mbar_init(&s.ring.full[k], 1);
            mbar_init(&s.ring.empty[k], W);
        }
        s.flag[0] = 0;
        s.flag[1] = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if ((threadIdx.x >> 5) == W) {
        if ((threadIdx.x & 31) == 0)
            producer<TYPE, STAGES>(s, p);
        return;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0)
        p.stamps[0] = global_ns();
    RowReduce rr{s.red, 0};
    Cursor cur;
    int occ = 0;
    for (int i = 0; i < p.n_tokens; i++) {
        const int pos = p.start_pos + i;
        int token = 0;
        if (i < p.n_prompt)
            token = p.prompt[i];
        else if (!next_token(s, p, i, token))
            break;
        bool ok = true;
        Trace tr;
        for (int l = 0; l < p.layers && ok; l++) {
            tr.open(p, occ++, 0);
            ok = phase_qkv<TYPE, STAGES>(s, p, tr, cur, rr, i, l, token, pos);
            tr.mark(7);
            if (!ok)
                break;
            tr.open(p, occ++, 1);
            ok = phase_att(s, p, tr, i, l, pos);
            tr.mark(7);
            if (!ok)
                break;
            tr.open(p, occ++, 2);
            ok = phase_wo<TYPE, STAGES>(s, p, tr, cur, rr, i, l, token);
            tr.mark(7);
            if (!ok)
                break;
            tr.open(p, occ++, 3);
            ok = phase_gu<TYPE, STAGES>(s, p, tr, cur, rr, i, l);
            tr.mark(7);
            if (!ok)
                break;
            tr.open(p, occ++, 4);
            ok = phase_down<TYPE, STAGES>(s, p, tr, cur, rr, i, l);
            tr.mark(7);
        }
        if (ok && wants_logits(p, i)) {
            tr.open(p, occ++, 5);
            ok = phase_lmhead<STAGES>(s, p, tr, cur, i);
            tr.mark(7);
        }
        if (!ok)
            break;
    }
    if (threadIdx.x == 0)
        atomicMax(p.stamps + 2, static_cast<unsigned long long>(global_ns()));
}

size_t fixed_smem(int stages, int dim, int ffn) {
    const int kmax = dim > ffn ? dim : ffn;
    size_t off = size_t(stages) * (kStageBytes + kStageScaleBytes);
    off += size_t(kmax) * 4;
    off = (off + 15) & ~size_t(15);
    return off;
}

/* Mirrors carve(): every piece after the union is 16-byte aligned. */
size_t tail_smem(int stages) {
    auto align16 = [](size_t o) { return (o + 15) & ~size_t(15); };
    size_t off = align16(2 * kRowBatch * W * 16 * 4);
    off = align16(off + W * 4);
    off = align16(off + W * 8);
    off = align16(off + 16);
    off = align16(off + 64 * 4);
    return off + size_t(stages) * 16 + 64; /* barriers, and slack */
}

/* Per-head attention scratch floats for a chunk of `ch` positions. */
size_t att_floats(int hd, int ch) {
    return size_t(hd) + 2 + NT + size_t(ch) * (2 * size_t(hd + 1) + 1);
}

template <int TYPE, int STAGES>
cudaError_t launch_t(MkParams p, int sms, size_t smem, cudaStream_t stream) {
    auto kernel = decode_mk_kernel<TYPE, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e != cudaSuccess)
        return e;
    void *args[] = {&p};
    nut::count_launches(1);
    return cudaLaunchCooperativeKernel(reinterpret_cast<void *>(kernel), dim3(sms),
                                       dim3(THREADS), args, smem, stream);
}

/* Picks the stage count and the union size for a shape: the most stages
 * (8, 6, 4) that leave room for the digits and at least 8 attention
 * positions per chunk. */
bool plan(int dim, int ffn, int hd, int nbmax, int max_smem, int &stages,
          size_t &union_bytes, int &chunk) {
    for (int st : {8, 6, 4}) {
        const size_t fixed = fixed_smem(st, dim, ffn) + tail_smem(st);
        if (fixed >= size_t(max_smem))
            continue;
        const size_t avail = (size_t(max_smem) - fixed) & ~size_t(15);
        if (avail < size_t(nbmax) * 136 || avail < att_floats(hd, 32) * 4)
            continue;
        stages = st;
        union_bytes = avail;
        chunk = int((avail / 4 - (size_t(hd) + 2 + NT)) / (2 * size_t(hd + 1) + 1));
        return true;
    }
    return false;
}

} // namespace

bool mk_supported(int dim, int ffn, int kvd, int head_dim, int heads, int type,
                  int max_smem) {
    (void)type;
    /* row tiles never straddle the q / k / v boundaries (dim and kv_dim
     * multiples of 16), every classifier row fits one stage */
    if (dim % 32 != 0 || ffn % 32 != 0 || kvd % 16 != 0 || dim * 4 > kStageBytes ||
        head_dim % 2 != 0 || head_dim > 256 || heads % (kvd / head_dim) != 0)
        return false;
    const int nb_dim = ((dim / 32) + 1) / 2 * 2, nb_ffn = ((ffn / 32) + 1) / 2 * 2;
    int stages, chunk;
    size_t ub;
    return plan(dim, ffn, head_dim, nb_dim > nb_ffn ? nb_dim : nb_ffn, max_smem, stages, ub,
                chunk);
}

cudaError_t launch_decode_mk(const MkParams &pin, int type, int sms, cudaStream_t stream) {
    int dev = 0, max_smem = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    MkParams p = pin;
    int stages = 0, chunk = 0;
    size_t ub = 0;
    const int nbmax = p.nb_dim > p.nb_ffn ? p.nb_dim : p.nb_ffn;
    if (!plan(p.dim, p.ffn, p.hd, nbmax, max_smem, stages, ub, chunk))
        return cudaErrorInvalidConfiguration;
    p.att_chunk = chunk;
    p.union_floats = int(ub / 4);
    const size_t smem = fixed_smem(stages, p.dim, p.ffn) + ub + tail_smem(stages);
    if (type == 1) {
        if (stages == 8)
            return launch_t<1, 8>(p, sms, smem, stream);
        if (stages == 6)
            return launch_t<1, 6>(p, sms, smem, stream);
        return launch_t<1, 4>(p, sms, smem, stream);
    }
    if (stages == 8)
        return launch_t<0, 8>(p, sms, smem, stream);
    if (stages == 6)
        return launch_t<0, 6>(p, sms, smem, stream);
    return launch_t<0, 4>(p, sms, smem, stream);
}

} // namespace nut
