/* The persistent token loop: every layer of every token of one generation
 * in a single cooperative launch (one CTA per SM).
 *
 * Per token i at position pos (reference decode_quantized_token,
 * src/quant_model.cpp:158-206, then the greedy head of generate_tokens_cached,
 * src/generate.cpp:197-205), for each layer l, three steps:
 *   QKV    x = rmsnorm(h) -> [q;k;v] = Wqkv x, RoPE on q and k
 *          (src/quant_model.cpp:26-37), k and v appended to the KV cache;
 *          CTAs own row tiles; q|k|v are published as tagged elements
 *   ATTWO  hA = h + Wo ctx, split by K: CTA (P, r) owns columns
 *          64 P .. 64 P + 63 of Wo (one pair of blocks) for the r-th share of
 *          its row tiles; it computes the GQA attention (src/quant_model.cpp:
 *          68-105) of the heads those columns cover and adds Wo[:, cols] ctx
 *          into an fp32 accumulator
 *   GUDOWN hB = hA + Wdown silu(Wgate x) * Wup x, x = rmsnorm(hA), split by
 *          FFN block: a CTA owns 32-unit blocks, computes their gate and up
 *          rows, the SwiGLU in shared memory, and adds Wdown[:, block] act
 *          into an fp32 accumulator
 * and, when the token's logits are needed, LMHEAD: x = rmsnorm(hB),
 * logits = W_cls x (fp32), argmax (first index of the maximum).
 *
 * Each CTA's weights form a fixed sequence of contiguous tile runs that its
 * producer warp streams through the shared-memory ring without ever waiting
 * for activations: weight traffic runs ahead across step and token
 * boundaries, limited only by the ring.
 *
 * Activations cross CTAs in two ways.  q|k|v travel as tagged vectors:
 * every element is written once per layer as one 64-bit (value, tag) store
 * and a consumer waits until each element it needs carries the expected
 * tag.  The residual stream travels through a ring of kAccSlots fp32
 * accumulators: the contributors of a step add their partial rows with
 * red.add, fence, and count themselves in the slot's counter; readers wait
 * (acquire) for the counter to reach the step's target and read the slot
 * through L2.  Step s (two per layer) uses slot s mod kAccSlots, whose
 * counter only grows, so step s's target is (s / kAccSlots + 1) times its
 * contributor count.  During step s every contributor zeroes its share of
 * slot s + 1 before counting itself, which orders the zeroing before every
 * red.add of step s + 1; the slot's previous readers (step s + 1 -
 * kAccSlots) finished long before, since each step waits for the last.
 * Float red.add makes the summation order of a step's partials vary from
 * run to run (parity is by tolerance, as for any reordered sum).
 * Key and value rows of the current position travel in the tagged q|k|v
 * vector; their cache stores precede a release store of the tag, and the
 * attention's acquire loads of those tags make every earlier cache store
 * of the same owner visible.  The next token id comes from a 64-bit
 * atomicMax key per token plus a count of CTAs that finished the
 * classifier.  Every wait is bounded by limit_ns and reports into *error.
 */
#include <algorithm>
#include <cmath>
#include <cstdio>

#include "decode_mk.h"
#include "kernels.h"
#include "stream.cuh"

namespace nut {
namespace {

constexpr int W = 8;             /* consumer warps (9 per CTA with the producer) */
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

/* Tag of the q|k|v elements of token i, layer l. */
__device__ __forceinline__ uint32_t qkv_tag(const MkParams &p, int i, int l) {
    return 1u + uint32_t(i * p.layers + l);
}

/* Accumulator steps: 2 per layer, kind 0 = hA (after ATTWO), 1 = hB (after
 * GUDOWN). */
__device__ __forceinline__ int step_of(const MkParams &p, int i, int l, int kind) {
    return 2 * (i * p.layers + l) + kind;
}
__device__ __forceinline__ float *slot_of(const MkParams &p, int step) {
    return p.hacc + size_t(step % kAccSlots) * p.dim;
}
__device__ __forceinline__ unsigned target_of(const MkParams &p, int step) {
    return unsigned(step / kAccSlots + 1) * unsigned((step & 1) ? p.count_gd : p.count_aw);
}

/* Range of part i in an even split of `total` into n parts
 * (total * n < 2^31 for every supported shape; 32-bit arithmetic avoids
 * the emulated 64-bit division). */
__device__ __forceinline__ void share_of(int total, int i, int n, int &a, int &b) {
    const unsigned t = unsigned(total), c = unsigned(n), k = unsigned(i);
    a = int(t * k / c);
    b = int(t * (k + 1) / c);
}
/* This CTA's range in an even split over the grid. */
__device__ __forceinline__ void share(int total, int &a, int &b) {
    share_of(total, int(blockIdx.x), int(gridDim.x), a, b);
}

struct Shared {
    Ring ring;
    float *xvec;       /* [kmax] staged activations */
    int8_t *dig;       /* union region: digits ... */
    float *fac;
    float *uni;        /* ... or attention scratch */
    float *red;        /* [2][kRowBatch][W][16] */
    float *part;       /* [2][W][kParkTiles][16] row-tile parks of the grouped path */
    float *wsum;       /* [W] */
    unsigned long long *bestk; /* [W] */
    int *flag;         /* [0] fatal, [1] token */
    float *yacc;       /* [dim] this CTA's partial rows of a split-K step */
    float *actv;       /* [kMaxFfnBlocks * 32] SwiGLU outputs of owned blocks */
};

/* Optional phase trace (thread 0 of each CTA): one record of kTraceWords
 * words per phase occurrence: phase id, the global timer at entry (1), and
 * SM clock stamps at entry (6), inputs staged (2), activation ready (3),
 * digits ready (4), weights consumed (5) and exit (7); sub-steps: the
 * finish's red.adds issued (8) and its fence passed (9), the gate/up tiles
 * consumed (11), the SwiGLU outputs complete
 * (12), and the key/value fence passed (13). */
struct Trace {
    unsigned long long *rec = nullptr;
    __device__ __forceinline__ void open(const MkParams &p, int occ, int id) {
        waited = 0;
        rec = p.trace != nullptr && occ < p.trace_stride
                  ? p.trace + (size_t(blockIdx.x) * p.trace_stride + occ) * kTraceWords
                  : nullptr;
        if (rec != nullptr && threadIdx.x == 0) {
            rec[0] = unsigned(id);
            rec[1] = global_ns();
            rec[6] = clock64();
        }
    }
    /* slots 2-5 and 7-15: SM clock (cycles) */
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
    s.part = reinterpret_cast<float *>(base + off);
    off = align16(off + size_t(2) * W * kParkTiles * 16 * 4);
    s.wsum = reinterpret_cast<float *>(base + off);
    off = align16(off + W * 4);
    s.bestk = reinterpret_cast<unsigned long long *>(base + off);
    off = align16(off + W * 8);
    s.flag = reinterpret_cast<int *>(base + off);
    off = align16(off + 16);
    s.yacc = reinterpret_cast<float *>(base + off);
    off = align16(off + size_t(p.dim + 32) * 4);
    s.actv = reinterpret_cast<float *>(base + off);
    off = align16(off + kMaxFfnBlocks * 32 * 4);
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

/* Waits for one tagged element.  The hand-off polls of this kernel spin
 * without sleeping between probes (one L2 round trip each, bounded by
 * `limit`): a sleep's granularity added to every hand-off (measured: 1,929
 * against 1,943 decode tok/s with the sleeps). */
template <bool ACQ>
__device__ __forceinline__ bool wait_tag(const Tagged *src, uint32_t tag,
                                         uint64_t limit, float &v) {
    uint64_t x = ACQ ? ld_acquire(src) : ld_relaxed(src);
    if (uint32_t(x >> 32) != tag) {
        const uint64_t t0 = global_ns();
        do {
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

constexpr int kPollBatch = 8; /* elements per thread of a staged vector */
constexpr int kResRegs = 2;   /* residual rows per thread held in registers */

/* Collective: waits until accumulator step `step` is complete (its counter
 * reached the step's target; thread 0 polls with acquire loads and the
 * barrier passes the ordering on).  The slot is then read with L2 loads
 * (__ldcg): lines of an older use of the slot may still sit in L1. */
__device__ bool wait_step(const Shared &s, const MkParams &p, int step) {
    if (threadIdx.x == 0) {
        const unsigned *c = p.cnt + step % kAccSlots;
        const unsigned want = target_of(p, step);
        if (ld_acquire_u32(c) < want) {
            const uint64_t t0 = global_ns();
            while (ld_acquire_u32(c) < want) {
                if (global_ns() - t0 > p.limit_ns) {
                    fatal(s, p, kErrTimeoutInput);
                    break;
                }
            }
        }
    }
    return healthy(s);
}

/* Collective: stages n (<= kPollBatch * NT) elements of a complete
 * accumulator slot into dst with the same thread mapping as NormW. */
__device__ void stage_slot(const float *src, int n, float *dst) {
#pragma unroll
    for (int j = 0; j < kPollBatch; j++) {
        const int k = threadIdx.x + j * NT;
        if (k < n)
            dst[k] = __ldcg(src + k);
    }
}

__device__ __forceinline__ void red_add4(float *dst, float4 v) {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(dst),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

/* Collective end of a contributor's share of accumulator step `step`:
 * adds yacc[0, nrows) into rows row0.. of the step's slot, zeroes this
 * contributor's share (index `me` of `count`) of the next step's slot, and
 * counts itself in.  The grid-barrier pattern: the CTA barrier orders every
 * thread's red.add and stores before thread 0's gpu-scope fence, which is
 * cumulative, so one fence ahead of the counter increment publishes them
 * all to any reader that acquires the counter. */
__device__ void finish_step(const Shared &s, const MkParams &p, int step, int row0, int nrows,
                            int me, int count, const Trace &tr) {
    cbar();
    float *dst = slot_of(p, step) + row0;
    const float4 *y4 = reinterpret_cast<const float4 *>(s.yacc);
    for (int k = threadIdx.x; k < nrows / 4; k += NT)
        red_add4(dst + 4 * k, y4[k]);
    int z0, z1;
    share_of(p.dim / 4, me, count, z0, z1);
    float4 *next = reinterpret_cast<float4 *>(slot_of(p, step + 1));
    for (int k = z0 + int(threadIdx.x); k < z1; k += NT)
        next[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    cbar();
    tr.mark(8);
    if (threadIdx.x == 0) {
        __threadfence();
        tr.mark(9);
        atomicAdd(p.cnt + step % kAccSlots, 1u);
    }
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

/* Blocks staged per round (per lane: one element each): every load of the
 * slice is issued before any is used, so the slice costs one L2 round trip
 * (one round for K <= 2 * W * 5 blocks, i.e. dim <= 4800). */
constexpr int kSliceBlocks = 10;

/* Element of the warp's k-th owned block: block index, or -1 past the end. */
__device__ __forceinline__ int slice_block(int w, int nb, int k) {
    const int p = w + (k >> 1) * W;
    return 2 * p < nb ? 2 * p + (k & 1) : -1;
}

/* Stages the warp's slice of an fp32 input vector of K elements (an
 * embedding row or a complete accumulator slot, read through L2), multiplies
 * it by `norm` (if any), writes its digits and block factors and returns
 * the lane's sum of squares of the raw inputs.  All loads are issued before
 * any is used and the block peaks are reduced together. */
template <int TYPE>
__device__ void warp_slice(const Shared &s, const float *src, int K, int nb,
                           const float *norm, float &ss) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float a_unit_inv = TYPE == 1 ? 1.0f / 16.0f : 1.0f;
    ss = 0.0f;
    for (int k0 = 0;; k0 += kSliceBlocks) {
        if (slice_block(w, nb, k0) < 0)
            break;
        float nw[kSliceBlocks], x[kSliceBlocks];
#pragma unroll
        for (int k = 0; k < kSliceBlocks; k++) {
            const int b = slice_block(w, nb, k0 + k), e = b * 32 + lane;
            const bool in = b >= 0 && e < K;
            nw[k] = norm != nullptr && in ? __ldg(norm + e) : 1.0f;
            x[k] = in ? __ldcg(src + e) : 0.0f;
        }
        uint32_t mb[kSliceBlocks];
#pragma unroll
        for (int k = 0; k < kSliceBlocks; k++) {
            ss = fmaf(x[k], x[k], ss);
            x[k] *= nw[k];
            mb[k] = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(x[k])));
        }
#pragma unroll
        for (int k = 0; k < kSliceBlocks; k++) {
            const int b = slice_block(w, nb, k0 + k);
            if (b >= 0)
                digit_from(x[k], mb[k], b, s.dig, s.fac, a_unit_inv);
        }
    }
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
    /* The input is hB of layer l - 1.  Layer 0 reads the embedding row, but
     * still waits for the previous token's last step: the q|k|v vector is
     * single-buffered, and that step completes only after every attention
     * of the previous token has read it. */
    const int prev = l > 0 ? step_of(p, i, l - 1, 1)
                           : (i > 0 ? step_of(p, i - 1, p.layers - 1, 1) : -1);
    if (prev >= 0 && !wait_step(s, p, prev))
        return false;
    const float *src = l == 0 ? p.emb + size_t(token) * p.dim
                              : slot_of(p, step_of(p, i, l - 1, 1));
    const int half = p.hd / 2;
    /* this position's RoPE row, staged for the epilogues (the first row-tile
     * barrier publishes it) */
    float *rope_cs = s.yacc, *rope_sn = s.yacc + half;
    float rc = 0.0f, rsn = 0.0f; /* loaded here, stored after the slice */
    if (int(threadIdx.x) < half) {
        rc = __ldg(p.rope_cos + size_t(pos) * half + threadIdx.x);
        rsn = __ldg(p.rope_sin + size_t(pos) * half + threadIdx.x);
    }
    float ss;
    warp_slice<TYPE>(s, src, p.dim, p.nb_dim, p.attn_norm + size_t(l) * p.dim, ss);
    slice_ss(s, ss);
    if (int(threadIdx.x) < half) {
        rope_cs[threadIdx.x] = rc;
        rope_sn[threadIdx.x] = rsn;
    }
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const TileRun run{L.qkv + size_t(a) * p.nb_dim * TB, L.qkv_s + size_t(a) * p.nb_dim * 16,
                      (b - a) * p.nb_dim, p.nb_dim};
    /* the grouped consume path gives warp w the pairs of warps w and w ^ 4
     * (W / 2 = 4): each digitised half of them */
    if (grouped_run<TYPE>(run))
        named_barrier(2 + ((threadIdx.x >> 5) & 3), 64);
    tr.mark(2);
    const uint32_t tag = qkv_tag(p, i, l);
    const int lane = threadIdx.x & 31;
    const float *cs = rope_cs, *sn = rope_sn;
    /* The cache rows of this token are read only by later tokens.  Each
     * lane that stored key/value rows fences once its tags are out (after
     * the run, off the path the attention waits on), which orders those
     * rows before the same lane's tags of the next token; the readers
     * acquire those tags (load, then fence) before fetching history. */
    bool wrote_kv = false;
    float nsc = -1.0f; /* the rmsnorm scale, computed at the first epilogue */
    auto epi = [&](int rt, float y) {
        if (nsc < 0.0f)
            nsc = norm_scale(s, p.dim);
        y *= nsc;
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
                st_relaxed(p.qkv + row, out, tag);
                p.kcache[((size_t(l) * p.kv_heads + h) * p.max_seq + pos) * p.hd + d] = out;
                wrote_kv = true;
            }
        } else if (lane < 16) {                   /* value */
            const int vr = row - p.dim - p.kvd, h = vr / p.hd, d = vr % p.hd;
            st_relaxed(p.qkv + row, y, tag);
            p.vcache[((size_t(l) * p.kv_heads + h) * p.max_seq + pos) * p.hd + d] = y;
            wrote_kv = true;
        }
    };
    const bool ok = consume_run<TYPE, W, STAGES>(s.ring, run, cur, s.dig, s.fac, rr,
                                                 threadIdx.x >> 5, kBar, epi,
                                                 tr.wait_acc());
    tr.mark(5);
    if (wrote_kv)
        __threadfence();
    tr.mark(13);
    tr.put_wait();
    return healthy(s) && ok;
}

/* Per-head attention scratch inside the union region. */
struct HeadScratch {
    float *q;        /* [hd] */
    float *wm, *wl;  /* [W] per-warp maximum and exp sum of a chunk */
    float *part;     /* [W][hd] per-warp partial contexts of a chunk */
    float *cur;      /* [2 hd] current k and v while pos is past the chunk */
    float *w;        /* [CH] exp weights */
    float *Kt, *Vt;  /* [CH][hd + 1] (padded rows: conflict-free) */
    int CH;
    __device__ HeadScratch(const Shared &s, const MkParams &p) {
        const int hd = p.hd, ld = hd + 1;
        q = s.uni;
        wm = q + hd;
        wl = wm + W;
        part = wl + W;
        cur = part + W * hd;
        w = cur + 2 * hd;
        const int used = hd + 2 * W + W * hd + 2 * hd;
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

/* Attention of query head h at position pos (attention_step,
 * src/quant_model.cpp:68-105: scores q.k / sqrt(hd), exp(score - max),
 * weights / total, context) over positions 0..pos in chunks of CH, with
 * the current q, k and v taken from the tagged q|k|v vector (tag tag_in):
 * the head's context vector into out[0, hd).  Within a chunk warp w takes
 * positions 32 w .. 32 w + 31 (one per lane): scores, the warp's maximum
 * and exp sum by shuffles, and its partial context (each lane owning dims
 * lane, lane + 32, ...); threads d < hd then merge the warps' partials into
 * a running (maximum, sum, context) carried across chunks.  Collective. */
__device__ bool head_context(const Shared &s, const MkParams &p, int l, int h, int pos,
                             uint32_t tag_in, float *out) {
    const int hd = p.hd, ld = hd + 1, G = p.heads / p.kv_heads;
    const float scale = 1.0f / sqrtf(float(hd));
    const HeadScratch t(s, p);
    const int g = h / G, lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
    /* history does not depend on this token: fetch it first */
    head_fetch(t, p, l, g, 0, min(t.CH, pos + 1), pos);
    /* q of head h and the current k, v of kv head g */
    if (threadIdx.x < 3 * hd) {
        const int part = threadIdx.x / hd, d = threadIdx.x - part * hd;
        const int row = part == 0 ? h * hd + d : p.dim + (part - 1) * p.kvd + g * hd + d;
        float v;
        if (wait_tag<false>(p.qkv + row, tag_in, p.limit_ns, v)) {
            if (part == 0)
                t.q[d] = v;
            else if (pos < t.CH)
                (part == 1 ? t.Kt : t.Vt)[pos * ld + d] = v;
            else
                t.cur[d + (part - 1) * hd] = v; /* kept for its chunk */
        } else {
            fatal(s, p, kErrTimeoutInput);
        }
    }
    __threadfence(); /* acquire: the tags order the older cache rows */
    if (!healthy(s)) {
        cp_async_wait_all();
        return false;
    }
    float m = -INFINITY, total = 0.0f, acc = 0.0f; /* running state of dim threadIdx.x */
    for (int p0 = 0; p0 <= pos; p0 += t.CH) {
        const int n = min(t.CH, pos + 1 - p0);
        if (p0 > 0) {
            head_fetch(t, p, l, g, p0, n, pos);
            if (pos >= p0 && pos < p0 + n && threadIdx.x < hd) {
                t.Kt[(pos - p0) * ld + threadIdx.x] = t.cur[threadIdx.x];
                t.Vt[(pos - p0) * ld + threadIdx.x] = t.cur[hd + threadIdx.x];
            }
        }
        cp_async_wait_all();
        cbar();
        const int j0 = 32 * wi, j = j0 + lane;
        if (j0 < n) {
            float sc = -INFINITY;
            if (j < n) {
                const float *kj = t.Kt + j * ld;
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
            const float mw = warp_max(sc);
            const float e = j < n ? expf(sc - mw) : 0.0f;
            const float lw = warp_sum(e);
            if (j < n)
                t.w[j] = e;
            __syncwarp();
            const int jn = min(32, n - j0);
            for (int d = lane; d < hd; d += 32) {
                const float *vj = t.Vt + j0 * ld + d;
                const float *ew = t.w + j0;
                float c = 0.0f;
                for (int k = 0; k < jn; k++)
                    c = fmaf(ew[k], vj[k * ld], c);
                t.part[wi * hd + d] = c;
            }
            if (lane == 0) {
                t.wm[wi] = mw;
                t.wl[wi] = lw;
            }
        }
        cbar();
        if (threadIdx.x < hd) {
            const int nw = (n + 31) / 32;
            float mc = m;
            for (int k = 0; k < nw; k++)
                mc = fmaxf(mc, t.wm[k]);
            const float f0 = expf(m - mc);
            float tn = total * f0, an = acc * f0;
            for (int k = 0; k < nw; k++) {
                const float f = expf(t.wm[k] - mc);
                tn = fmaf(t.wl[k], f, tn);
                an = fmaf(t.part[k * hd + threadIdx.x], f, an);
            }
            m = mc;
            total = tn;
            acc = an;
        }
        cbar(); /* tiles and partials are reused by the next chunk */
    }
    if (threadIdx.x < hd)
        out[threadIdx.x] = acc / total;
    cbar();
    return true;
}

/* ---- attention of long histories (the LONG kernel) ---------------------

   Generations whose positions exceed one attention chunk run a second
   instantiation of the kernel with the functions below; the others keep
   the single-chunk code above unchanged (the persistent kernel's speed
   depends on its register allocation and code layout, measured: folding
   both into one instantiation cost 2-12 % at short contexts). */

/* Per-head attention scratch of the LONG kernel.  Key and value rows
 * are padded to hd + 4 floats: 16-byte rows for the bulk of the copies,
 * and a float4 read by the 8 lanes of a quarter-warp (8 consecutive
 * positions) touches 8 distinct 16-byte bank groups. */
struct LongScratch {
    float *q;        /* [hd] */
    float *wm, *wl;  /* [W] per-warp maximum and exp sum of a chunk */
    float *part;     /* [W][hd] per-warp partial contexts of a chunk */
    float *cur;      /* [2 hd] current k and v while pos is past the chunk */
    float *w;        /* [CH] exp weights */
    float *Kt, *Vt;  /* [CH][hd + 4] */
    int CH, ld;
    __device__ LongScratch(const Shared &s, const MkParams &p) {
        const int hd = p.hd;
        ld = hd + 4;
        q = s.uni;
        wm = q + hd;
        wl = wm + W;
        part = wl + W;
        cur = part + W * hd;
        w = cur + 2 * hd;
        const int used = hd + 2 * W + W * hd + 2 * hd + 3; /* + padding of w */
        CH = (p.union_floats - used) / (2 * ld + 1);
        if (CH > NT)
            CH = NT;
        Kt = w + ((CH + 3) & ~3);
        Vt = Kt + CH * ld;
    }
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}

/* Asynchronous copies of cached keys and values of kv head g, positions
 * [p0, p0 + n) other than `pos`, into the tiles (16 bytes per copy; hd is a
 * multiple of 4). */
__device__ __forceinline__ void long_fetch(const LongScratch &t, const MkParams &p, int l,
                                           int g, int p0, int n, int pos) {
    const int hd = p.hd, q4 = hd / 4;
    const size_t base = (size_t(l) * p.kv_heads + g) * size_t(p.max_seq) * hd;
    for (int idx = threadIdx.x; idx < n * q4; idx += NT) {
        const int j = idx / q4, d = (idx - j * q4) * 4, q = p0 + j;
        if (q == pos)
            continue;
        const size_t off = base + size_t(q) * hd + d;
        cp_async16(t.Kt + j * t.ld + d, p.kcache + off);
        cp_async16(t.Vt + j * t.ld + d, p.vcache + off);
    }
}

/* Partial attention of query head h at position pos (attention_step,
 * src/quant_model.cpp:68-105: scores q.k / sqrt(hd), exp(score - max),
 * weights / total, context) over positions lo .. hi of the history (hi <=
 * pos), in chunks of CH, with q, and the current k and v when hi == pos,
 * taken from the tagged q|k|v vector (tag tag_in).  Threads d < hd return
 * the running maximum m, the exp sum `total` and the unnormalised context
 * `acc` of dim d (context = acc / total).  Within a chunk warp w takes
 * positions 32 w .. 32 w + 31 (one per lane): scores, the warp's maximum
 * and exp sum by shuffles, and its partial context (each lane owning dims
 * lane, lane + 32, ...); threads d < hd then merge the warps' partials into
 * the running state carried across chunks.  Collective. */
__device__ bool head_partial(const Shared &s, const MkParams &p, int l, int h, int pos,
                             uint32_t tag_in, int lo, int hi, float &m, float &total,
                             float &acc) {
    const int hd = p.hd, G = p.heads / p.kv_heads;
    const float scale = 1.0f / sqrtf(float(hd));
    const LongScratch t(s, p);
    const int ld = t.ld;
    const int g = h / G, lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
    /* history does not depend on this token: fetch it first */
    long_fetch(t, p, l, g, lo, min(t.CH, hi + 1 - lo), pos);
    /* q of head h and, when this range ends at pos, the current k, v of kv
     * head g */
    const bool has_cur = hi == pos;
    if (threadIdx.x < 3 * hd) {
        const int part = threadIdx.x / hd, d = threadIdx.x - part * hd;
        if (part == 0 || has_cur) {
            const int row = part == 0 ? h * hd + d : p.dim + (part - 1) * p.kvd + g * hd + d;
            float v;
            if (wait_tag<false>(p.qkv + row, tag_in, p.limit_ns, v)) {
                if (part == 0)
                    t.q[d] = v;
                else if (pos - lo < t.CH)
                    (part == 1 ? t.Kt : t.Vt)[(pos - lo) * ld + d] = v;
                else
                    t.cur[d + (part - 1) * hd] = v; /* kept for its chunk */
            } else {
                fatal(s, p, kErrTimeoutInput);
            }
        }
    }
    __threadfence(); /* acquire: the tags order the older cache rows */
    if (!healthy(s)) {
        cp_async_wait_all();
        return false;
    }
    m = -INFINITY, total = 0.0f, acc = 0.0f; /* running state of dim threadIdx.x */
    for (int p0 = lo; p0 <= hi; p0 += t.CH) {
        const int n = min(t.CH, hi + 1 - p0);
        if (p0 > lo) {
            long_fetch(t, p, l, g, p0, n, pos);
            if (pos >= p0 && pos < p0 + n && threadIdx.x < hd) {
                t.Kt[(pos - p0) * ld + threadIdx.x] = t.cur[threadIdx.x];
                t.Vt[(pos - p0) * ld + threadIdx.x] = t.cur[hd + threadIdx.x];
            }
        }
        cp_async_wait_all();
        cbar();
        const int j0 = 32 * wi, j = j0 + lane;
        if (j0 < n) {
            float sc = -INFINITY;
            if (j < n) {
                const float4 *k4 = reinterpret_cast<const float4 *>(t.Kt + j * ld);
                const float4 *q4 = reinterpret_cast<const float4 *>(t.q);
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                for (int d = 0; d < hd / 4; d++) {
                    const float4 kk = k4[d], qq = q4[d];
                    a0 = fmaf(qq.x, kk.x, a0);
                    a1 = fmaf(qq.y, kk.y, a1);
                    a2 = fmaf(qq.z, kk.z, a2);
                    a3 = fmaf(qq.w, kk.w, a3);
                }
                sc = ((a0 + a1) + (a2 + a3)) * scale;
            }
            const float mw = warp_max(sc);
            const float e = j < n ? expf(sc - mw) : 0.0f;
            const float lw = warp_sum(e);
            if (j < n)
                t.w[j] = e;
            __syncwarp();
            const int jn = min(32, n - j0);
            for (int d = lane; d < hd; d += 32) {
                const float *vj = t.Vt + j0 * ld + d;
                const float *ew = t.w + j0;
                float c = 0.0f;
                for (int k = 0; k < jn; k++)
                    c = fmaf(ew[k], vj[k * ld], c);
                t.part[wi * hd + d] = c;
            }
            if (lane == 0) {
                t.wm[wi] = mw;
                t.wl[wi] = lw;
            }
        }
        cbar();
        if (threadIdx.x < hd) {
            const int nw = (n + 31) / 32;
            float mc = m;
            for (int k = 0; k < nw; k++)
                mc = fmaxf(mc, t.wm[k]);
            const float f0 = expf(m - mc);
            float tn = total * f0, an = acc * f0;
            for (int k = 0; k < nw; k++) {
                const float f = expf(t.wm[k] - mc);
                tn = fmaf(t.wl[k], f, tn);
                an = fmaf(t.part[k * hd + threadIdx.x], f, an);
            }
            m = mc;
            total = tn;
            acc = an;
        }
        cbar(); /* tiles and partials are reused by the next chunk */
    }
    return true;
}

/* Whether the cpp CTAs of a block pair split head attention by positions
 * at position pos: when the history needs more than one chunk, the pair's
 * 64 columns lie inside one head (hd a multiple of 64), there is more than
 * one CTA per pair, every share holds a position, and the merge's
 * [cpp][hd + 2] states fit the key tile.  Every CTA decides the same. */
__device__ __forceinline__ bool split_history(const Shared &s, const MkParams &p, int pos) {
    const LongScratch t(s, p);
    return p.cpp > 1 && p.hd % 64 == 0 && pos + 1 > t.CH && pos + 1 >= p.cpp &&
           p.cpp * (p.hd + 2) <= t.CH * t.ld;
}

/* Combines the partial states of the cpp CTAs of block pair P (each over its
 * share of the positions) into the head's context out[0, hd): this CTA's
 * state (threads d < hd: m, total, acc) is published as tagged elements
 * [acc[0..hd), m, total] in slot P cpp + part of p.xchg, the other CTAs'
 * states are read as their tags arrive, and every CTA merges them in slot
 * order (m = max m_k, total = sum total_k e^(m_k - m), context = sum acc_k
 * e^(m_k - m) / total), so the pair's CTAs compute the same context.
 * Collective. */
__device__ bool merge_history(const Shared &s, const MkParams &p, int P, int part,
                              uint32_t tag, float m, float total, float acc, float *out) {
    const int hd = p.hd, E = hd + 2, cpp = p.cpp;
    const LongScratch t(s, p);
    float *X = t.Kt; /* [cpp][E]: the tiles are free after head_partial */
    Tagged *mine = p.xchg + size_t(P * cpp + part) * E;
    if (int(threadIdx.x) < hd) {
        st_relaxed(mine + threadIdx.x, acc, tag);
        X[part * E + threadIdx.x] = acc;
        if (threadIdx.x == 0) {
            st_relaxed(mine + hd, m, tag);
            st_relaxed(mine + hd + 1, total, tag);
            X[part * E + hd] = m;
            X[part * E + hd + 1] = total;
        }
    }
    for (int idx = threadIdx.x; idx < cpp * E; idx += NT) {
        const int k = idx / E;
        if (k == part)
            continue;
        float v;
        if (wait_tag<false>(p.xchg + size_t(P * cpp) * E + idx, tag, p.limit_ns, v))
            X[idx] = v;
        else
            fatal(s, p, kErrTimeoutInput);
    }
    if (!healthy(s))
        return false;
    if (int(threadIdx.x) < hd) {
        float M = -INFINITY;
        for (int k = 0; k < cpp; k++)
            M = fmaxf(M, X[k * E + hd]);
        float L = 0.0f, c = 0.0f;
        for (int k = 0; k < cpp; k++) {
            const float f = expf(X[k * E + hd] - M);
            L = fmaf(X[k * E + hd + 1], f, L);
            c = fmaf(X[k * E + threadIdx.x], f, c);
        }
        out[threadIdx.x] = c / L;
    }
    cbar(); /* X is reused by the next head */
    return true;
}

/* ATTWO (hA = h + Wo ctx), split by K: CTA c < count_aw owns the block pair
 * P = c / cpp (ctx columns 64 P .. 64 P + 63) for share c mod cpp of Wo's
 * row tiles.  It computes the attention of every head those columns cover
 * (a head may be computed by several CTAs), multiplies its Wo tiles, adds
 * the residual rows when P == 0, and adds its rows into step 2 (i L + l). */
template <int TYPE, int STAGES, bool LONG>
__device__ bool phase_attwo(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                            int i, int l, int token, int pos) {
    const int c = blockIdx.x;
    if (c >= p.count_aw)
        return true;
    const int P = c / p.cpp, part = c - P * p.cpp;
    int a, b;
    share_of(p.rt_wo, part, p.cpp, a, b);
    const int st = step_of(p, i, l, 0);
    const uint32_t tag_in = qkv_tag(p, i, l);
    /* P == 0 adds the residual rows: the embedding row at layer 0, else hB of
     * layer l - 1.  Their loads are issued first and land during the
     * attention; rows past kResRegs * NT (only when cpp is small) are read
     * at the end. */
    const int nrows = (b - a) * 16;
    const float *res = nullptr;
    float resv[kResRegs];
    if (P == 0) {
        if (l > 0 && !wait_step(s, p, st - 1))
            return false;
        res = (l == 0 ? p.emb + size_t(token) * p.dim : slot_of(p, st - 1)) + a * 16;
#pragma unroll
        for (int j = 0; j < kResRegs; j++) {
            const int r = int(threadIdx.x) + j * NT;
            resv[j] = r < nrows ? __ldcg(res + r) : 0.0f;
        }
    }
    float *xs = s.xvec, *hc = s.xvec + 64;
    const int e0 = 64 * P;
    if (threadIdx.x < 64)
        xs[threadIdx.x] = 0.0f;
    const int h0 = e0 / p.hd, h1 = min(p.heads - 1, (e0 + 63) / p.hd);
    /* LONG: past one chunk of history the pair's CTAs take equal shares of
     * the positions and merge their partial states (h0 == h1 then) */
    bool split = false;
    int lo = 0, hi = pos;
    if constexpr (LONG) {
        split = split_history(s, p, pos);
        if (split) {
            lo = int(unsigned(pos + 1) * unsigned(part) / unsigned(p.cpp));
            hi = int(unsigned(pos + 1) * unsigned(part + 1) / unsigned(p.cpp)) - 1;
        }
    }
    for (int h = h0; h <= h1; h++) {
        if constexpr (LONG) {
            float m, total, acc;
            if (!head_partial(s, p, l, h, pos, tag_in, lo, hi, m, total, acc))
                return false;
            if (split) {
                if (!merge_history(s, p, P, part, tag_in, m, total, acc, hc))
                    return false;
            } else {
                if (int(threadIdx.x) < p.hd)
                    hc[threadIdx.x] = acc / total;
                cbar();
            }
        } else {
            if (!head_context(s, p, l, h, pos, tag_in, hc))
                return false;
        }
        if (threadIdx.x < 64) {
            const int e = e0 + threadIdx.x;
            if (e < p.dim && e / p.hd == h)
                xs[threadIdx.x] = hc[e - h * p.hd];
        }
        cbar();
    }
    tr.mark(2);
    const int w = threadIdx.x >> 5;
    if (w < 2)
        digit_block(xs, 64, w, s.dig, s.fac, TYPE == 1 ? 1.0f / 16.0f : 1.0f);
    cbar();
    tr.mark(4);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const size_t t0 = (size_t(P) * p.rt_wo + a) * 2;
    const TileRun run{L.wo + t0 * TB, L.wo_s + t0 * 16, (b - a) * 2, 2};
    const bool ok = consume_cols<TYPE, W, STAGES, true>(s.ring, run, cur, s.dig, s.fac, 1,
                                                        s.yacc, w, tr.wait_acc());
    tr.mark(5);
    tr.put_wait();
    if (P == 0) {
        cbar(); /* every row of yacc written */
#pragma unroll
        for (int j = 0; j < kResRegs; j++) {
            const int r = int(threadIdx.x) + j * NT;
            if (r < nrows)
                s.yacc[r] += resv[j];
        }
        for (int r = int(threadIdx.x) + kResRegs * NT; r < nrows; r += NT)
            s.yacc[r] += __ldcg(res + r);
    }
    finish_step(s, p, st, a * 16, nrows, c, p.count_aw, tr);
    return healthy(s) && ok;
}

/* The FFN step's work, split evenly over the CTAs.  Each 32-unit block b
 * is U = gd_unit work units: its 4 gate/up row tiles 4 b .. 4 b + 3 (row
 * tiles of the interleaved matrix, 8 units each), then its Wdown column
 * block in units of kDownUnitPairs row-tile pairs.  CTA c takes the
 * contiguous unit range [u0, u1) of the nbf U units.  A block's Wdown
 * units need all 32 SwiGLU outputs of the block, so gate/up tiles whose
 * block's Wdown is (partly) owned by a later CTA are "exported": published
 * as tagged values; only the first Wdown block of a range can "import"
 * tiles computed by earlier CTAs.  The gate/up tiles are consumed as one
 * run in tile order (measured: one run with its exported tiles last beats
 * an exported-first run followed by the rest, 1,945 against 1,938 decode
 * tok/s, since each run pays its own start-up, barrier and epilogue). */
struct GdPlan {
    int gu_lo, gu_hi; /* gate/up row tiles [gu_lo, gu_hi) */
    int ex_lo;        /* exported tiles [ex_lo, gu_hi) */
    int d_lo, d_hi;   /* Wdown units [d_lo, d_hi) (block d / du, part d % du) */
    int du;           /* Wdown units per block */
    int db_lo, nd;    /* Wdown blocks db_lo .. db_lo + nd - 1 (digit slots) */
};

__device__ __forceinline__ GdPlan gd_plan(const MkParams &p, int c) {
    const int U = p.gd_unit, du = U - 4;
    int u0, u1;
    share_of(p.gd_total, c, int(gridDim.x), u0, u1);
    GdPlan g;
    g.du = du;
    /* gate/up tiles and Wdown units among units [0, u) */
    auto gu_before = [&](int u) { return 4 * (u / U) + min(u % U, 4); };
    auto d_before = [&](int u) { return du * (u / U) + max(u % U - 4, 0); };
    g.gu_lo = gu_before(u0);
    g.gu_hi = gu_before(u1);
    g.d_lo = d_before(u0);
    g.d_hi = d_before(u1);
    g.ex_lo = g.gu_hi;
    if (g.gu_hi > g.gu_lo) {
        const int bl = (g.gu_hi - 1) / 4; /* block of the last gate/up tile */
        if ((bl + 1) * du > g.d_hi)
            g.ex_lo = max(g.gu_lo, 4 * bl);
    }
    g.db_lo = g.d_lo / du;
    g.nd = g.d_hi > g.d_lo ? (g.d_hi - 1) / du - g.db_lo + 1 : 0;
    return g;
}

/* GUDOWN (hB = hA + Wdown silu(gate) * up) over this CTA's work units: its
 * gate/up tiles, SwiGLU (src/quant_model.cpp:197-198) into shared memory
 * (and, for exported tiles, into the tagged act vector), then its Wdown
 * units, plus its share of the residual rows, added into step 2 (i L + l)
 * + 1. */
template <int TYPE, int STAGES>
__device__ bool phase_gudown(const Shared &s, const MkParams &p, Trace &tr, Cursor &cur,
                             RowReduce &rr, int i, int l) {
    const int c = blockIdx.x;
    if (c >= p.count_gd)
        return true;
    const GdPlan g = gd_plan(p, c);
    const int st = step_of(p, i, l, 1);
    if (!wait_step(s, p, st - 1))
        return false;
    const float *hA = slot_of(p, st - 1);
    /* this CTA's share of the residual rows, loaded alongside the slice */
    int r0, r1;
    share_of(p.dim / 16, c, p.count_gd, r0, r1);
    float resv[kResRegs];
#pragma unroll
    for (int j = 0; j < kResRegs; j++) {
        const int r = r0 * 16 + int(threadIdx.x) + j * NT;
        resv[j] = r < r1 * 16 ? __ldcg(hA + r) : 0.0f;
    }
    float ss = 0.0f;
    if (g.gu_hi > g.gu_lo)
        warp_slice<TYPE>(s, hA, p.dim, p.nb_dim, p.ffn_norm + size_t(l) * p.dim, ss);
    slice_ss(s, ss);
    for (int r = threadIdx.x; r < p.dim + 32; r += NT)
        s.yacc[r] = 0.0f;
    cbar(); /* zeroing and the residual rows use different thread mappings */
#pragma unroll
    for (int j = 0; j < kResRegs; j++) {
        const int r = r0 * 16 + int(threadIdx.x) + j * NT;
        if (r < r1 * 16)
            s.yacc[r] = resv[j];
    }
    for (int r = r0 * 16 + int(threadIdx.x) + kResRegs * NT; r < r1 * 16; r += NT)
        s.yacc[r] = __ldcg(hA + r);
    tr.mark(2);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const MkLayerPtrs &L = p.layer[l];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t tag = qkv_tag(p, i, l);
    /* tile t: lanes 0-7 gate rows, lanes 8-15 up rows of units 8 t .. 8 t + 7 */
    float nsc = -1.0f; /* the rmsnorm scale, computed at the first epilogue */
    int t_first = 0;   /* first tile of the run being consumed */
    auto epi = [&](int rt, float y) {
        if (nsc < 0.0f)
            nsc = norm_scale(s, p.dim);
        y *= nsc;
        const float up = __shfl_down_sync(0xffffffffu, y, 8);
        const int t = t_first + rt, b = t >> 2, unit = 8 * (t & 3) + lane;
        if (lane < 8) {
            const float a = y / (1.0f + expf(-y)) * up;
            if (b >= g.db_lo && b < g.db_lo + g.nd)
                s.actv[(b - g.db_lo) * 32 + unit] = a;
            if (t >= g.ex_lo)
                st_relaxed(p.act + 32 * b + unit, a, tag);
        }
    };
    bool ok = true;
    if (g.gu_hi > g.gu_lo) {
        t_first = g.gu_lo;
        const TileRun gu{L.gu + size_t(g.gu_lo) * p.nb_dim * TB,
                         L.gu_s + size_t(g.gu_lo) * p.nb_dim * 16,
                         (g.gu_hi - g.gu_lo) * p.nb_dim, p.nb_dim};
        ok = consume_run<TYPE, W, STAGES>(s.ring, gu, cur, s.dig, s.fac, rr, w, kBar, epi,
                                          tr.wait_acc());
    }
    tr.mark(11);
    cbar(); /* every SwiGLU output written; the gate/up digits are free */
    tr.mark(12);
    if (w < g.nd) {
        /* digits of Wdown block db_lo + w; tiles before gu_lo come from
         * earlier CTAs through the tagged vector */
        const int b = g.db_lo + w, t = 4 * b + (lane >> 3);
        float v = 0.0f;
        if (t < g.gu_lo) {
            if (!wait_tag<false>(p.act + 32 * b + lane, tag, p.limit_ns, v))
                fatal(s, p, kErrTimeoutInput);
        } else {
            v = s.actv[w * 32 + lane];
        }
        digit_from(v, __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))), w, s.dig,
                   s.fac, TYPE == 1 ? 1.0f / 16.0f : 1.0f);
    }
    if (!healthy(s))
        return false;
    tr.mark(4);
    for (int d = g.d_lo; d < g.d_hi; d++) {
        const int b = d / g.du, part = d - b * g.du, slot = b - g.db_lo;
        const int q0 = part * kDownUnitPairs;
        const int np = min(kDownUnitPairs, p.rt_down_pairs - q0);
        const size_t t0 = size_t(b) * size_t(2 * p.rt_down_pairs) + size_t(2 * q0);
        const TileRun down{L.down + t0 * TB, L.down_s + t0 * 16, 2 * np, 1};
        ok = consume_cols<TYPE, W, STAGES, false>(s.ring, down, cur, s.dig + slot * 128,
                                                  s.fac + 2 * slot, np, s.yacc + 32 * q0, w,
                                                  tr.wait_acc()) &&
             ok;
    }
    tr.mark(5);
    tr.put_wait();
    finish_step(s, p, st, 0, p.dim, c, p.count_gd, tr);
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
        const int last = step_of(p, i, p.layers - 1, 1);
        if (!wait_step(s, p, last))
            return false;
        stage_slot(slot_of(p, last), p.dim, s.xvec);
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
    const int c = blockIdx.x;
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
            if (c < p.count_aw) {
                const int P = c / p.cpp;
                share_of(p.rt_wo, c - P * p.cpp, p.cpp, a, b);
                const size_t t0 = (size_t(P) * p.rt_wo + a) * 2;
                if (!produce_run_c<TYPE, STAGES>(s.ring,
                        TileRun{L.wo + t0 * TB, L.wo_s + t0 * 16, (b - a) * 2, 2}, cur))
                    return;
            }
            if (c < p.count_gd) {
                /* the consumer's order: the gate/up tiles, then the Wdown
                 * units */
                const GdPlan g = gd_plan(p, c);
                if (g.gu_hi > g.gu_lo &&
                    !produce_run_c<TYPE, STAGES>(s.ring,
                        TileRun{L.gu + size_t(g.gu_lo) * p.nb_dim * TB,
                                L.gu_s + size_t(g.gu_lo) * p.nb_dim * 16,
                                (g.gu_hi - g.gu_lo) * p.nb_dim, p.nb_dim}, cur))
                    return;
                for (int d = g.d_lo; d < g.d_hi; d++) {
                    const int b = d / g.du, q0 = (d - b * g.du) * kDownUnitPairs;
                    const int np = min(kDownUnitPairs, p.rt_down_pairs - q0);
                    const size_t t0 = size_t(b) * size_t(2 * p.rt_down_pairs) + size_t(2 * q0);
                    if (!produce_run_c<TYPE, STAGES>(s.ring,
                            TileRun{L.down + t0 * TB, L.down_s + t0 * 16, 2 * np, 1}, cur))
                        return;
                }
            }
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

template <int TYPE, int STAGES, bool LONG>
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
    RowReduce rr{s.red, 0, s.part, 0};
    Cursor cur;
    int occ = 0;
    bool alive = true;
    for (int i = 0; i < p.n_tokens; i++) {
        const int pos = p.start_pos + i;
        int token = 0;
        if (i < p.n_prompt)
            token = p.prompt[i];
        else if (!next_token(s, p, i, token)) {
            alive = false;
            break;
        }
        bool ok = true;
        Trace tr;
        for (int l = 0; l < p.layers && ok; l++) {
            tr.open(p, occ++, 0);
            ok = phase_qkv<TYPE, STAGES>(s, p, tr, cur, rr, i, l, token, pos);
            tr.mark(7);
            if (!ok)
                break;
            tr.open(p, occ++, 1);
            ok = phase_attwo<TYPE, STAGES, LONG>(s, p, tr, cur, i, l, token, pos);
            tr.mark(7);
            if (!ok)
                break;
            tr.open(p, occ++, 2);
            ok = phase_gudown<TYPE, STAGES>(s, p, tr, cur, rr, i, l);
            tr.mark(7);
        }
        if (ok && wants_logits(p, i)) {
            tr.open(p, occ++, 5);
            ok = phase_lmhead<STAGES>(s, p, tr, cur, i);
            tr.mark(7);
        }
        if (!ok) {
            alive = false;
            break;
        }
    }
    /* the last hidden vector (hB of the last layer of the last token) */
    if (alive && blockIdx.x == 0) {
        const int last = step_of(p, p.n_tokens - 1, p.layers - 1, 1);
        if (wait_step(s, p, last))
            for (int k = threadIdx.x; k < p.dim; k += NT)
                p.hidden_out[k] = __ldcg(slot_of(p, last) + k);
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
size_t tail_smem(int stages, int dim) {
    auto align16 = [](size_t o) { return (o + 15) & ~size_t(15); };
    size_t off = align16(2 * kRowBatch * W * 16 * 4);
    off = align16(off + size_t(2) * W * kParkTiles * 16 * 4);
    off = align16(off + W * 4);
    off = align16(off + W * 8);
    off = align16(off + 16);
    off = align16(off + size_t(dim + 32) * 4);
    off = align16(off + kMaxFfnBlocks * 32 * 4);
    return off + size_t(stages) * 16 + 64; /* barriers, and slack */
}

/* Per-head attention scratch floats for a chunk of `ch` positions (mirrors
 * HeadScratch). */
size_t att_floats(int hd, int ch) {
    return size_t(hd) * (3 + W) + 2 * W + 3 + size_t(ch) * (2 * size_t(hd + 4) + 1);
}

template <int TYPE, int STAGES, bool LONG>
cudaError_t launch_t(MkParams p, int sms, size_t smem, cudaStream_t stream) {
    auto kernel = decode_mk_kernel<TYPE, STAGES, LONG>;
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
        const size_t fixed = fixed_smem(st, dim, ffn) + tail_smem(st, dim);
        if (fixed >= size_t(max_smem))
            continue;
        const size_t avail = (size_t(max_smem) - fixed) & ~size_t(15);
        if (avail < size_t(nbmax) * 136 || avail < att_floats(hd, 32) * 4)
            continue;
        stages = st;
        union_bytes = avail;
        chunk = int((avail / 4 - (size_t(hd) * (3 + W) + 2 * W + 3)) / (2 * size_t(hd + 4) + 1));
        return true;
    }
    return false;
}

} // namespace

bool mk_supported(int dim, int ffn, int kvd, int head_dim, int heads, int type,
                  int max_smem, int sms) {
    (void)type;
    /* row tiles never straddle the q / k / v boundaries (dim and kv_dim
     * multiples of 16), every classifier row fits one stage, the staging
     * vector holds a context pair and one head, and no CTA owns more FFN
     * blocks than kMaxFfnBlocks */
    if (dim % 32 != 0 || ffn % 32 != 0 || kvd % 16 != 0 || dim * 4 > kStageBytes ||
        head_dim % 2 != 0 || head_dim > 256 || heads % (kvd / head_dim) != 0 ||
        dim < 64 + head_dim || sms <= 0)
        return false;
    /* the FFN step's unit ranges touch at most kMaxFfnBlocks blocks */
    const int rt_down = (dim / 16 + 1) / 2 * 2;
    const int U = ffn_units_per_block(rt_down / 2);
    const int per_cta = (ffn / 32 * U + sms - 1) / sms;
    if ((per_cta + U - 1) / U + 1 > kMaxFfnBlocks)
        return false;
    /* every Wo block pair needs its own CTA (the step counts them all) */
    if ((dim / 32 + 1) / 2 > sms)
        return false;
    const int nb_dim = ((dim / 32) + 1) / 2 * 2, nb_ffn = ((ffn / 32) + 1) / 2 * 2;
    int stages, chunk;
    size_t ub;
    return plan(dim, ffn, head_dim, nb_dim > nb_ffn ? nb_dim : nb_ffn, max_smem, stages, ub,
                chunk);
}

namespace {
template <bool LONG>
cudaError_t launch_type(const MkParams &p, int type, int stages, int sms, size_t smem,
                        cudaStream_t stream) {
    if (type == 1) {
        if (stages == 8)
            return launch_t<1, 8, LONG>(p, sms, smem, stream);
        if (stages == 6)
            return launch_t<1, 6, LONG>(p, sms, smem, stream);
        return launch_t<1, 4, LONG>(p, sms, smem, stream);
    }
    if (stages == 8)
        return launch_t<0, 8, LONG>(p, sms, smem, stream);
    if (stages == 6)
        return launch_t<0, 6, LONG>(p, sms, smem, stream);
    return launch_t<0, 4, LONG>(p, sms, smem, stream);
}
} // namespace

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
    const size_t smem = fixed_smem(stages, p.dim, p.ffn) + ub + tail_smem(stages, p.dim);
    /* the LONG kernel when some pass of this launch attends to more
     * positions than one chunk holds (and its 16-byte copies apply) */
    const int chunk_short = int((ub / 4 - (size_t(p.hd) * (3 + W) + 2 * W)) /
                                (2 * size_t(p.hd + 1) + 1));
    const bool lng = p.hd % 4 == 0 && p.start_pos + p.n_tokens > std::min(chunk_short, NT);
    if (lng)
        return launch_type<true>(p, type, stages, sms, smem, stream);
    return launch_type<false>(p, type, stages, sms, smem, stream);
}

} // namespace nut
