#pragma once
/* Weight streaming and the tensor-pipe quantised dot products.
 *
 * A producer warp streams contiguous runs of fragment tiles (tiles.h) from
 * HBM into a ring of shared-memory stages with bulk asynchronous copies
 * (cp.async.bulk, completion counted on an mbarrier).  Consumer warps wait
 * for a stage, multiply its tiles against the activation vector with
 * mma.sync.m16n8k32 (s8 x s8 -> s32) and release it.
 *
 * Activations enter the tensor pipe as exact integer digits: per
 * 32-element block b with peak |x| in [2^e, 2^(e+1)), x is scaled by the
 * power of two 2^(25-e) and rounded to an integer V (|V| < 2^26, error
 * <= 2^-26 of the block peak), then split into four signed 7-bit digits,
 * V = d1 2^21 + d2 2^14 + d3 2^7 + d4.  The B operand of one mma carries
 * the four digits of one block in four of its eight columns (columns 0-3
 * for even blocks, 4-7 for odd blocks), so a pair of mma's on blocks
 * (b, b+1) fills all eight columns with exact int32 block sums
 * D_{r,b,d} = sum_k A[r][k] d_d[k].  Accumulators start at the bit pattern
 * of 1.5 * 2^23, so each exact sum |D| < 2^22 is read back as a float with
 * one subtraction.  The epilogue folds digits, the activation scale and
 * the weight block scale into fp32:
 *   y_r += s[r,b] * E_b 2^-27 / A_unit * (D1 2^21 + D2 2^14 + D3 2^7 + D4)
 * with A_unit = 16 for INT4 (nibbles are widened to 16 q) and 1 for INT8.
 */
#include <cstdint>
#include <cuda_fp16.h>

#include "common.cuh"

namespace nut {

/* ---- PTX wrappers -------------------------------------------------- */

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar))
                 : "memory");
}

/* Arrival that counts `count` times (one warp standing in for several). */
__device__ __forceinline__ void mbar_arrive_n(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

/* Waits for the phase with `parity` to complete; false after `limit_ns`.
 * Between probes the warp sleeps, so waiting warps leave the issue slots
 * to the warps that have work. */
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t start = global_ns();
    for (;;) {
        __nanosleep(32);
        if (mbar_try_wait(bar, parity))
            return true;
        if (global_ns() - start > limit_ns)
            return false;
    }
}

/* Bulk copy global -> this CTA's shared memory, completing on `bar`.
 * Addresses 16-byte aligned, size a multiple of 16. */
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1], %2, [%3];\n" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4],
                                       uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

/* ---- ring of stages ------------------------------------------------ */

constexpr int kStageBytes = 16384;     /* data bytes per stage */
constexpr int kStageScaleBytes = 2048; /* scale bytes per stage (64 tiles) */
constexpr int kMagic = 0x4B400000;     /* bits of 1.5 * 2^23 */
constexpr float kMagicF = 12582912.0f;

enum : int {
    kErrNone = 0,
    kErrTimeoutFull = 1,  /* a consumer gave up waiting for weights */
    kErrTimeoutEmpty = 2, /* the producer gave up waiting for a free stage */
    kErrTimeoutInput = 3, /* a consumer gave up waiting for its input vector */
};

struct Ring {
    uint8_t *data;      /* [stages][kStageBytes] */
    uint16_t *scales;   /* [stages][kStageScaleBytes / 2] */
    uint64_t *full;     /* [stages] */
    uint64_t *empty;    /* [stages] */
    int stages;
    uint64_t limit_ns;
    int *error;         /* global error word */
    int *fatal;         /* shared flag: a consumer gave up; the others stop
                           waiting but keep the barrier sequence */
};

__device__ __forceinline__ void report(int *error, int code) {
    atomicCAS(error, 0, code);
}

/* One contiguous run of fragment tiles (this CTA's row tiles of one
 * matrix): tiles [0, tiles) at data / scales, blocks per row tile nb. */
struct TileRun {
    const uint8_t *data;
    const uint16_t *scales;
    int tiles;
    int nb;
};

template <int TYPE> struct TileGeom {
    static constexpr int kTileBytes = TYPE == 0 ? 512 : 256;
    static constexpr int kChunkTiles = kStageBytes / kTileBytes; /* 32 / 64 */
};

/* Producer side: issues the run's chunks; `chunk` counts stages used by
 * this CTA so far and is advanced.  Returns false on timeout. */
template <int TYPE>
__device__ bool produce_run(const Ring &ring, const TileRun &run, uint32_t &chunk) {
    using G = TileGeom<TYPE>;
    for (int t = 0; t < run.tiles; t += G::kChunkTiles) {
        const int n = min(G::kChunkTiles, run.tiles - t);
        const int stage = int(chunk % uint32_t(ring.stages));
        const uint32_t parity = ((chunk / uint32_t(ring.stages)) & 1u) ^ 1u;
        if (!mbar_wait(&ring.empty[stage], parity, ring.limit_ns)) {
            report(ring.error, kErrTimeoutEmpty);
            return false;
        }
        const uint32_t db = uint32_t(n * G::kTileBytes), sb = uint32_t(n * 32);
        mbar_expect_tx(&ring.full[stage], db + sb);
        bulk_g2s(ring.data + size_t(stage) * kStageBytes,
                 run.data + size_t(t) * G::kTileBytes, db, &ring.full[stage]);
        bulk_g2s(ring.scales + size_t(stage) * (kStageScaleBytes / 2),
                 run.scales + size_t(t) * 16, sb, &ring.full[stage]);
        chunk++;
    }
    return true;
}

/* fp32 run (rows of `row_bytes`, chunked by whole rows). */
__device__ __forceinline__ bool produce_bytes(const Ring &ring, const uint8_t *src,
                                              size_t bytes, uint32_t chunk_bytes,
                                              uint32_t &chunk) {
    for (size_t off = 0; off < bytes; off += chunk_bytes) {
        const uint32_t n = uint32_t(min(size_t(chunk_bytes), bytes - off));
        const int stage = int(chunk % uint32_t(ring.stages));
        const uint32_t parity = ((chunk / uint32_t(ring.stages)) & 1u) ^ 1u;
        if (!mbar_wait(&ring.empty[stage], parity, ring.limit_ns)) {
            report(ring.error, kErrTimeoutEmpty);
            return false;
        }
        mbar_expect_tx(&ring.full[stage], n);
        bulk_g2s(ring.data + size_t(stage) * kStageBytes, src + off, n,
                 &ring.full[stage]);
        chunk++;
    }
    return true;
}

/* ---- activation digits --------------------------------------------- */

/* Digits of x (K values, zero padded to nb blocks) into dig[nb][4][32]
 * and the per-block factors fac[nb][2] = {E 2^-13, E 2^-27} / a_unit.
 * Called by all `warps` consumer warps (warp index w); the block peak is
 * one redux.sync over the magnitudes' bit patterns (order-preserving for
 * non-negative floats). */
/* Digits of block b from the lane's value v and the block's peak bits
 * (the redux of |v| over the warp), for callers that batch the reduxes. */
__device__ __forceinline__ void digit_from(float v, uint32_t mbits, int b, int8_t *dig,
                                           float *fac, float a_unit_inv) {
    const int lane = threadIdx.x & 31;
    const float m = __uint_as_float(mbits);
    int d1 = 0, d2 = 0, d3 = 0, d4 = 0;
    float f_hi = 0.0f, f_lo = 0.0f;
    if (m >= 0x1p-100f) {
        const int e = int((mbits >> 23) & 0xff) - 127;
        const float up = __uint_as_float(uint32_t(25 - e + 127) << 23);
        int V = __float2int_rn(v * up);
        d4 = ((V + 64) & 127) - 64;
        V = (V - d4) >> 7;
        d3 = ((V + 64) & 127) - 64;
        V = (V - d3) >> 7;
        d2 = ((V + 64) & 127) - 64;
        d1 = (V - d2) >> 7;
        /* E = 2^(e+2): E 2^-13 and E 2^-27 are exact powers of two */
        f_hi = __uint_as_float(uint32_t(e + 2 - 13 + 127) << 23) * a_unit_inv;
        f_lo = __uint_as_float(uint32_t(e + 2 - 27 + 127) << 23) * a_unit_inv;
    }
    int8_t *db = dig + b * 128;
    db[lane] = int8_t(d1);
    db[32 + lane] = int8_t(d2);
    db[64 + lane] = int8_t(d3);
    db[96 + lane] = int8_t(d4);
    if (lane == 0) {
        fac[2 * b] = f_hi;
        fac[2 * b + 1] = f_lo;
    }
}

__device__ __forceinline__ void digit_block(const float *x, int K, int b, int8_t *dig,
                                            float *fac, float a_unit_inv) {
    const int k = b * 32 + (threadIdx.x & 31);
    const float v = k < K ? x[k] : 0.0f;
    digit_from(v, __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))), b, dig, fac,
               a_unit_inv);
}

__device__ __forceinline__ void make_digits(const float *x, int K, int nb, int w,
                                            int warps, int8_t *dig, float *fac,
                                            float a_unit_inv) {
    int b = w;
    for (; b + warps < nb; b += 2 * warps) {
        digit_block(x, K, b, dig, fac, a_unit_inv);
        digit_block(x, K, b + warps, dig, fac, a_unit_inv);
    }
    if (b < nb)
        digit_block(x, K, b, dig, fac, a_unit_inv);
}

/* ---- consuming a run ------------------------------------------------- */

/* d = A x B + (1.5 * 2^23 as int32): the constant accumulator seed that
 * lets each exact int32 block sum be read back as a float. */
__device__ __forceinline__ void mma_s8_seeded(int (&d)[4], const uint32_t (&a)[4],
                                              uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
          "r"(kMagic));
}

template <int TYPE>
__device__ __forceinline__ void load_a(const uint8_t *stage_data, int tile,
                                       uint32_t (&a)[4]) {
    const int lane = threadIdx.x & 31;
    if (TYPE == 0) {
        const uint4 p =
            *reinterpret_cast<const uint4 *>(stage_data + size_t(tile) * 512 + 16 * lane);
        a[0] = p.x, a[1] = p.y, a[2] = p.z, a[3] = p.w;
    } else {
        const uint2 p =
            *reinterpret_cast<const uint2 *>(stage_data + size_t(tile) * 256 + 8 * lane);
        a[0] = (p.x << 4) & 0xF0F0F0F0u, a[1] = p.x & 0xF0F0F0F0u;
        a[2] = (p.y << 4) & 0xF0F0F0F0u, a[3] = p.y & 0xF0F0F0F0u;
    }
}

/* Dot products of one block pair (tiles `tile`, `tile` + 1 of the stage,
 * blocks b0, b0 + 1) accumulated into the lane's partial sums for rows g
 * and g + 8.  The two mma's are independent: columns 0-3 of the first and
 * 4-7 of the second carry the digits. */
template <int TYPE>
__device__ __forceinline__ void pair_mma(const uint8_t *stage_data,
                                         const uint16_t *stage_scales, int tile,
                                         int b0, const int8_t *dig,
                                         const float *fac, float &yg, float &yg8) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    uint32_t a0[4], a1[4];
    load_a<TYPE>(stage_data, tile, a0);
    load_a<TYPE>(stage_data, tile + 1, a1);
    const int slot = g >> 2, half = c >> 1;
    const int8_t *src = dig + (b0 + slot) * 128 + (g & 3) * 32 + 4 * c;
    const uint32_t bx0 = *reinterpret_cast<const uint32_t *>(src);
    const uint32_t bx1 = *reinterpret_cast<const uint32_t *>(src + 16);
    int d0[4], d1[4];
    mma_s8_seeded(d0, a0, slot == 0 ? bx0 : 0u, slot == 0 ? bx1 : 0u);
    mma_s8_seeded(d1, a1, slot == 1 ? bx0 : 0u, slot == 1 ? bx1 : 0u);
    const int e0 = half ? d1[0] : d0[0], e1 = half ? d1[1] : d0[1];
    const int e2 = half ? d1[2] : d0[2], e3 = half ? d1[3] : d0[3];
    const float f0 = __int_as_float(e0) - kMagicF, f1 = __int_as_float(e1) - kMagicF;
    const float f2 = __int_as_float(e2) - kMagicF, f3 = __int_as_float(e3) - kMagicF;
    const float tg = fmaf(f0, 128.0f, f1), tg8 = fmaf(f2, 128.0f, f3);
    const float F = fac[2 * (b0 + half) + (c & 1)];
    const uint16_t *sc = stage_scales + (tile + half) * 16;
    yg = fmaf(tg, half_bits_to_float(sc[g]) * F, yg);
    yg8 = fmaf(tg8, half_bits_to_float(sc[g + 8]) * F, yg8);
}

/* Finished row tiles are reduced in batches of this many: their shuffle
 * chains interleave and a batch costs one barrier instead of one per row
 * tile. */
constexpr int kRowBatch = 4;

/* Row tiles parked per chunk by the grouped consume path. */
constexpr int kParkTiles = 16;

/* Per-CTA reduction buffers for row-tile results. */
struct RowReduce {
    float *red;  /* [2][kRowBatch][warps][16] (general path) */
    int buf;
    float *part; /* [2][warps][kParkTiles][16] (grouped path), or null */
    int pbuf;    /* half of `part` the next grouped run uses */
};

/* Runs that consume_run hands to the grouped path (when it has a park
 * buffer): row tiles of whole stages. */
template <int TYPE>
__device__ __forceinline__ bool grouped_run(const TileRun &run) {
    constexpr int CT = TileGeom<TYPE>::kChunkTiles;
    return run.nb % CT == 0 && run.tiles % run.nb == 0;
}

/* Stage cursor: the CTA-wide count of consumed stages, kept as (index,
 * parity) so no division is needed. */
struct Cursor {
    int stage = 0;
    uint32_t parity = 0;
    template <int STAGES> __device__ __forceinline__ void next() {
        if (++stage == STAGES) {
            stage = 0;
            parity ^= 1u;
        }
    }
};

/* Reduces the batch's n finished row tiles (first index rt_first): lanes
 * c of a row group, then the warps in a fixed-order tree; row tile k of
 * the batch is finished on warp k % WARPS, which calls epi(rt, y) with y
 * on lanes 0..15. */
template <int WARPS, typename Epi>
__device__ __forceinline__ void flush_rows(float (&sg)[kRowBatch], float (&sg8)[kRowBatch],
                                           int n, int rt_first, RowReduce &rr, int w,
                                           int barrier_id, Epi &epi) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int k = 0; k < kRowBatch; k++) {
        sg[k] += __shfl_xor_sync(0xffffffffu, sg[k], 1);
        sg8[k] += __shfl_xor_sync(0xffffffffu, sg8[k], 1);
    }
#pragma unroll
    for (int k = 0; k < kRowBatch; k++) {
        sg[k] += __shfl_xor_sync(0xffffffffu, sg[k], 2);
        sg8[k] += __shfl_xor_sync(0xffffffffu, sg8[k], 2);
    }
    float *red = rr.red + rr.buf * kRowBatch * WARPS * 16;
    if (c == 0) {
#pragma unroll
        for (int k = 0; k < kRowBatch; k++) {
            red[(k * WARPS + w) * 16 + g] = sg[k];
            red[(k * WARPS + w) * 16 + g + 8] = sg8[k];
        }
    }
    named_barrier(barrier_id, WARPS * 32);
    for (int k = w; k < n; k += WARPS) {
        const float *rk = red + k * WARPS * 16;
        float v[WARPS];
#pragma unroll
        for (int j = 0; j < WARPS; j++)
            v[j] = lane < 16 ? rk[j * 16 + (lane & 15)] : 0.0f;
#pragma unroll
        for (int step = 1; step < WARPS; step *= 2)
#pragma unroll
            for (int j = 0; j + step < WARPS; j += 2 * step)
                v[j] += v[j + step];
        epi(rt_first + k, v[0]);
    }
    rr.buf ^= 1;
}

/* Products of one pair of tiles (tiles `tile`, `tile` + 1 of the stage,
 * blocks b0, b0 + 1) as pair_mma computes them, with the two mma's chained
 * into one accumulator: the first product's B carries block b0's digits
 * only in columns 0-3 and the second's block b0 + 1's only in columns 4-7,
 * so D = A1 B1 + (A0 B0 + seed) holds exactly pair_mma's column sums and
 * every lane reads its two digit sums from one result.  Writes (does not
 * add) the lane's partial sums for rows g and g + 8. */
template <int TYPE>
__device__ __forceinline__ void pair_chain(const uint8_t *stage_data,
                                           const uint16_t *stage_scales, int tile,
                                           int b0, const int8_t *dig,
                                           const float *fac, float &yg, float &yg8) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    uint32_t a0[4], a1[4];
    load_a<TYPE>(stage_data, tile, a0);
    load_a<TYPE>(stage_data, tile + 1, a1);
    const int slot = g >> 2, half = c >> 1;
    const int8_t *src = dig + (b0 + slot) * 128 + (g & 3) * 32 + 4 * c;
    const uint32_t bx0 = *reinterpret_cast<const uint32_t *>(src);
    const uint32_t bx1 = *reinterpret_cast<const uint32_t *>(src + 16);
    const uint32_t m = slot == 0 ? 0xffffffffu : 0u;
    int d[4];
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0[0]), "r"(a0[1]), "r"(a0[2]), "r"(a0[3]), "r"(bx0 & m), "r"(bx1 & m),
          "r"(kMagic));
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a1[0]), "r"(a1[1]), "r"(a1[2]), "r"(a1[3]), "r"(bx0 & ~m), "r"(bx1 & ~m));
    const float f0 = __int_as_float(d[0]) - kMagicF, f1 = __int_as_float(d[1]) - kMagicF;
    const float f2 = __int_as_float(d[2]) - kMagicF, f3 = __int_as_float(d[3]) - kMagicF;
    const float tg = fmaf(f0, 128.0f, f1), tg8 = fmaf(f2, 128.0f, f3);
    const float F = fac[2 * (b0 + half) + (c & 1)];
    const uint16_t *sc = stage_scales + (tile + half) * 16;
    yg = tg * (half_bits_to_float(sc[g]) * F);
    yg8 = tg8 * (half_bits_to_float(sc[g + 8]) * F);
}

/* consume_run for runs whose row tiles are whole stages (nb a multiple of
 * a stage's tiles), when rr.part is given.  The WARPS consumer warps form
 * two groups of WARPS / 2: group q takes the run's stages q, q + 2, ..., so
 * one group's per-stage tail overlaps the other's products, and warp gw of
 * a group multiplies the stage's pairs gw, gw + WARPS / 2, ... (block pairs
 * congruent to gw modulo WARPS / 2: a warp needs the digits of its own
 * pairs and of warp gw + WARPS / 2's, which callers make visible) into
 * independent accumulators.  Each warp parks its sum of every row tile in
 * its own slots of rr.part (shuffles over the four lanes of a row group,
 * then one add per row), in stage order; after every kParkTiles row tiles
 * (and at the end) one barrier, then warp k finishes row tiles k, k +
 * WARPS, ... of the chunk: y = the warps' parks added in warp order (a fixed
 * order), epi(rt, y) with y on lanes 0..15, as in flush_rows. */
template <int TYPE, int WARPS, int STAGES, typename Epi>
__device__ bool consume_rows_grouped(const Ring &ring, const TileRun &run, Cursor &cur,
                                     const int8_t *dig, const float *fac, float *part, int w,
                                     int barrier_id, Epi &epi, long long *wait_cycles) {
    using G = TileGeom<TYPE>;
    constexpr int GW = WARPS / 2;               /* warps per group */
    static_assert(WARPS == 2 * GW, "two groups of equal size");
    constexpr int PP = G::kChunkTiles / 2 / GW; /* pairs per warp per stage */
    static_assert(PP * 2 * GW == G::kChunkTiles, "stage split");
    const int group = w / GW, gw = w % GW;
    const int lane = threadIdx.x & 31;
    const int spr = run.nb / G::kChunkTiles; /* stages per row tile */
    const int nrt = run.tiles / run.nb;
    float *mine = part + size_t(w) * kParkTiles * 16;
    bool poisoned = false;
    for (int c0 = 0; c0 < nrt; c0 += kParkTiles) {
        const int c1 = min(nrt, c0 + kParkTiles);
        if (lane < 16)
            for (int r = 0; r < c1 - c0; r++)
                mine[r * 16 + lane] = 0.0f;
        __syncwarp();
        for (int j = c0 * spr + group; j < c1 * spr; j += 2) {
            const int idx = cur.stage + j;
            const int stage = idx % STAGES;
            const uint32_t parity = cur.parity ^ (uint32_t(idx / STAGES) & 1u);
            if (!poisoned)
                poisoned = *reinterpret_cast<volatile int *>(ring.fatal) != 0;
            const long long w0 = wait_cycles != nullptr ? clock64() : 0;
            if (!poisoned && !mbar_wait(&ring.full[stage], parity, ring.limit_ns)) {
                report(ring.error, kErrTimeoutFull);
                *reinterpret_cast<volatile int *>(ring.fatal) = 1;
                poisoned = true;
            }
            if (wait_cycles != nullptr)
                *wait_cycles += clock64() - w0;
            if (!poisoned) {
                const uint8_t *sd = ring.data + size_t(stage) * kStageBytes;
                const uint16_t *ss = ring.scales + size_t(stage) * (kStageScaleBytes / 2);
                const int kb = (j % spr) * G::kChunkTiles; /* first block of the stage */
                float y[PP], y8[PP];
#pragma unroll
                for (int u = 0; u < PP; u++) {
                    const int tl = 2 * (gw + u * GW);
                    pair_chain<TYPE>(sd, ss, tl, kb + tl, dig, fac, y[u], y8[u]);
                }
                float t = y[0], t8 = y8[0];
#pragma unroll
                for (int u = 1; u < PP; u++) {
                    t += y[u];
                    t8 += y8[u];
                }
                t += __shfl_xor_sync(0xffffffffu, t, 1);
                t8 += __shfl_xor_sync(0xffffffffu, t8, 1);
                t += __shfl_xor_sync(0xffffffffu, t, 2);
                t8 += __shfl_xor_sync(0xffffffffu, t8, 2);
                if ((lane & 3) == 0) {
                    const int r = j / spr - c0, g = lane >> 2;
                    mine[r * 16 + g] += t;
                    mine[r * 16 + g + 8] += t8;
                }
            }
            __syncwarp();
            /* the ring's stages expect WARPS arrivals: each of the group's
             * WARPS / 2 warps counts twice */
            if (lane == 0 && !poisoned)
                mbar_arrive_n(&ring.empty[stage], 2);
        }
        named_barrier(barrier_id, WARPS * 32); /* every park of the chunk written */
        for (int r = w; r < c1 - c0; r += WARPS) {
            float v = 0.0f;
            if (lane < 16) {
#pragma unroll
                for (int q = 0; q < WARPS; q++)
                    v += part[(size_t(q) * kParkTiles + r) * 16 + lane];
            }
            epi(c0 + r, v);
        }
        if (c1 < nrt)
            named_barrier(barrier_id, WARPS * 32); /* parks free for the next chunk */
    }
    /* every consumer passes the run's stages */
    const int nst = nrt * spr;
    const int idx = cur.stage + nst;
    cur.parity ^= uint32_t(idx / STAGES) & 1u;
    cur.stage = idx % STAGES;
    return !poisoned;
}

/* Consumes one run of row tiles with WARPS consumer warps (w = this warp).
 * Every finished row tile `rt` (index within the run) reaches epi(rt, y)
 * on one warp, lanes 0..15 holding y for rows 16 rt + lane (other lanes
 * hold 0), in batches of kRowBatch.  Returns false on timeout; all
 * consumer warps take the same path. */
template <int TYPE, int WARPS, int STAGES, bool ROTATE = false, typename Epi>
__device__ bool consume_run(const Ring &ring, const TileRun &run, Cursor &cur,
                            const int8_t *dig, const float *fac, RowReduce &rr,
                            int w, int barrier_id, Epi &&epi,
                            long long *wait_cycles = nullptr) {
    using G = TileGeom<TYPE>;
    if constexpr (WARPS % 2 == 0 && (G::kChunkTiles / 2) % (WARPS / 2) == 0) {
        if (rr.part != nullptr && grouped_run<TYPE>(run)) {
            /* consecutive runs alternate halves: a warp may zero its slots
             * for run n + 1 while a slower warp still reads run n's (it
             * cannot reach run n + 2 before run n + 1's barrier) */
            float *half = rr.part + size_t(rr.pbuf) * WARPS * kParkTiles * 16;
            rr.pbuf ^= 1;
            return consume_rows_grouped<TYPE, WARPS, STAGES>(ring, run, cur, dig, fac, half, w,
                                                             barrier_id, epi, wait_cycles);
        }
    }
    const int lane = threadIdx.x & 31;
    float ya = 0.0f, ya8 = 0.0f, yb = 0.0f, yb8 = 0.0f;
    float sg[kRowBatch], sg8[kRowBatch];
#pragma unroll
    for (int k = 0; k < kRowBatch; k++)
        sg[k] = sg8[k] = 0.0f;
    int nslot = 0, batch_first = 0;
    const int nb = run.nb;
    int rt = 0, rt_base = 0; /* current row tile and its first tile index */
    bool poisoned = false;
    for (int t = 0; t < run.tiles; t += G::kChunkTiles) {
        const int n = min(G::kChunkTiles, run.tiles - t);
        if (!poisoned)
            poisoned = *reinterpret_cast<volatile int *>(ring.fatal) != 0;
        const long long w0 = wait_cycles != nullptr ? clock64() : 0;
        if (!poisoned && !mbar_wait(&ring.full[cur.stage], cur.parity, ring.limit_ns)) {
            report(ring.error, kErrTimeoutFull);
            *reinterpret_cast<volatile int *>(ring.fatal) = 1;
            poisoned = true;
        }
        if (wait_cycles != nullptr)
            *wait_cycles += clock64() - w0;
        const uint8_t *sd = ring.data + size_t(cur.stage) * kStageBytes;
        const uint16_t *ss = ring.scales + size_t(cur.stage) * (kStageScaleBytes / 2);
        const int end = t + n;
        while (rt_base < end) {
            const int lo = max(t, rt_base), hi = min(end, rt_base + nb);
            /* pairs of this row tile inside [lo, hi) owned by warp w.  By
             * default pair p of every row tile belongs to warp p mod WARPS,
             * so a warp always uses the same activation blocks: callers
             * whose warps digitise only their own blocks (and start without
             * a CTA barrier) rely on this.  With ROTATE (every block's
             * digits written before a barrier), pair q of the run
             * (q = rt_base / 2 + p) belongs to warp q mod WARPS instead, so
             * the remainder pairs of consecutive row tiles land on
             * different warps. */
            const int p_lo = (lo - rt_base) >> 1, p_hi = (hi - rt_base) >> 1;
            const int q_lo = ROTATE ? (rt_base >> 1) + p_lo : p_lo;
            int p = p_lo + ((w - q_lo % WARPS) + WARPS) % WARPS;
            if (poisoned)
                p = p_hi;
            for (; p + WARPS < p_hi; p += 2 * WARPS) {
                pair_mma<TYPE>(sd, ss, rt_base + 2 * p - t, 2 * p, dig, fac, ya, ya8);
                pair_mma<TYPE>(sd, ss, rt_base + 2 * (p + WARPS) - t, 2 * (p + WARPS),
                               dig, fac, yb, yb8);
            }
            if (p < p_hi)
                pair_mma<TYPE>(sd, ss, rt_base + 2 * p - t, 2 * p, dig, fac, ya, ya8);
            if (rt_base + nb > end)
                break; /* row tile continues in the next stage */
            /* row tile finished for this warp: park it in its batch slot */
#pragma unroll
            for (int k = 0; k < kRowBatch; k++)
                if (k == nslot) {
                    sg[k] = ya + yb;
                    sg8[k] = ya8 + yb8;
                }
            ya = ya8 = yb = yb8 = 0.0f;
            if (++nslot == kRowBatch) {
                flush_rows<WARPS>(sg, sg8, nslot, batch_first, rr, w, barrier_id, epi);
                nslot = 0;
                batch_first = rt + 1;
            }
            rt++;
            rt_base += nb;
        }
        __syncwarp();
        if (lane == 0 && !poisoned)
            mbar_arrive(&ring.empty[cur.stage]);
        cur.template next<STAGES>();
    }
    if (nslot > 0) {
#pragma unroll
        for (int k = 0; k < kRowBatch; k++)
            if (k >= nslot)
                sg[k] = sg8[k] = 0.0f;
        flush_rows<WARPS>(sg, sg8, nslot, batch_first, rr, w, barrier_id, epi);
    }
    return !poisoned;
}

/* ---- consuming a column-split run ------------------------------------

   Runs of the pair-column and block-column tile orders: the CTA owns a
   K slice of one or two blocks per row tile, so a row tile's product is
   finished inside one pair and needs no reduction across warps.  Pair q of
   the run is tiles (2q, 2q+1):
     SAME_ROW (pair-column): both tiles are row tile q, blocks 0 and 1 of
       `dig`; the B operand carries block 0's digits in columns 0-3 and
       block 1's in 4-7, and the four lanes c of a row group sum to row
       tile q's rows.  yacc[16 q + r] = result.
     !SAME_ROW (block-column): pair q covers row tiles 2 lq and 2 lq + 1
       (lq = q mod pairs_per_block) of block k = q / pairs_per_block; both
       halves of B carry block k's digits, lanes c = 0, 1 sum row tile 2 lq
       and lanes c = 2, 3 row tile 2 lq + 1.  yacc[16 (2 lq + h) + r] +=
       result (blocks accumulate).
   Warp (SAME_ROW ? q : lq) mod WARPS handles pair q, so every yacc row has
   a single writer.  Returns false on timeout. */
template <int TYPE, bool SAME_ROW>
__device__ __forceinline__ void pair_cols(const uint8_t *stage_data,
                                          const uint16_t *stage_scales, int tile,
                                          int blk0, int blk1, const int8_t *dig,
                                          const float *fac, float &yg, float &yg8) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3, half = c >> 1;
    uint32_t a0[4], a1[4];
    load_a<TYPE>(stage_data, tile, a0);
    load_a<TYPE>(stage_data, tile + 1, a1);
    const int8_t *src = dig + (g < 4 ? blk0 : blk1) * 128 + (g & 3) * 32 + 4 * c;
    const uint32_t bx0 = *reinterpret_cast<const uint32_t *>(src);
    const uint32_t bx1 = *reinterpret_cast<const uint32_t *>(src + 16);
    int d0[4], d1[4];
    mma_s8_seeded(d0, a0, bx0, bx1);
    mma_s8_seeded(d1, a1, bx0, bx1);
    const int e0 = half ? d1[0] : d0[0], e1 = half ? d1[1] : d0[1];
    const int e2 = half ? d1[2] : d0[2], e3 = half ? d1[3] : d0[3];
    const float f0 = __int_as_float(e0) - kMagicF, f1 = __int_as_float(e1) - kMagicF;
    const float f2 = __int_as_float(e2) - kMagicF, f3 = __int_as_float(e3) - kMagicF;
    const float tg = fmaf(f0, 128.0f, f1), tg8 = fmaf(f2, 128.0f, f3);
    const float F = fac[2 * (half ? blk1 : blk0) + (c & 1)];
    const uint16_t *sc = stage_scales + (tile + half) * 16;
    yg = tg * (half_bits_to_float(sc[g]) * F);
    yg8 = tg8 * (half_bits_to_float(sc[g + 8]) * F);
}

template <int TYPE, int WARPS, int STAGES, bool SAME_ROW>
__device__ bool consume_cols(const Ring &ring, const TileRun &run, Cursor &cur,
                             const int8_t *dig, const float *fac, int pairs_per_block,
                             float *yacc, int w, long long *wait_cycles = nullptr) {
    using G = TileGeom<TYPE>;
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    bool poisoned = false;
    for (int t = 0; t < run.tiles; t += G::kChunkTiles) {
        const int n = min(G::kChunkTiles, run.tiles - t);
        if (!poisoned)
            poisoned = *reinterpret_cast<volatile int *>(ring.fatal) != 0;
        const long long w0 = wait_cycles != nullptr ? clock64() : 0;
        if (!poisoned && !mbar_wait(&ring.full[cur.stage], cur.parity, ring.limit_ns)) {
            report(ring.error, kErrTimeoutFull);
            *reinterpret_cast<volatile int *>(ring.fatal) = 1;
            poisoned = true;
        }
        if (wait_cycles != nullptr)
            *wait_cycles += clock64() - w0;
        const uint8_t *sd = ring.data + size_t(cur.stage) * kStageBytes;
        const uint16_t *ss = ring.scales + size_t(cur.stage) * (kStageScaleBytes / 2);
        const int q0 = t >> 1, q1 = (t + n) >> 1;
        if (!poisoned) {
            if (SAME_ROW) {
                for (int q = q0 + ((w - q0 % WARPS) + WARPS) % WARPS; q < q1; q += WARPS) {
                    float y, y8;
                    pair_cols<TYPE, true>(sd, ss, 2 * q - t, 0, 1, dig, fac, y, y8);
                    y += __shfl_xor_sync(0xffffffffu, y, 1);
                    y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
                    y += __shfl_xor_sync(0xffffffffu, y, 2);
                    y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
                    if (c == 0) {
                        yacc[16 * q + g] = y;
                        yacc[16 * q + g + 8] = y8;
                    }
                }
            } else {
                for (int k = q0 / pairs_per_block; k * pairs_per_block < q1; k++) {
                    const int base = k * pairs_per_block;
                    const int lo = max(q0 - base, 0), hi = min(q1 - base, pairs_per_block);
                    for (int lq = lo + ((w - lo % WARPS) + WARPS) % WARPS; lq < hi;
                         lq += WARPS) {
                        float y, y8;
                        pair_cols<TYPE, false>(sd, ss, 2 * (base + lq) - t, k, k, dig, fac,
                                               y, y8);
                        y += __shfl_xor_sync(0xffffffffu, y, 1);
                        y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
                        if ((c & 1) == 0) {
                            const int row = 16 * (2 * lq + (c >> 1)) + g;
                            yacc[row] += y;
                            yacc[row + 8] += y8;
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && !poisoned)
            mbar_arrive(&ring.empty[cur.stage]);
        cur.template next<STAGES>();
    }
    return !poisoned;
}

/* Producer counterpart of consume_run. */
template <int TYPE, int STAGES>
__device__ bool produce_run_c(const Ring &ring, const TileRun &run, Cursor &cur) {
    using G = TileGeom<TYPE>;
    for (int t = 0; t < run.tiles; t += G::kChunkTiles) {
        const int n = min(G::kChunkTiles, run.tiles - t);
        if (!mbar_wait(&ring.empty[cur.stage], cur.parity ^ 1u, ring.limit_ns)) {
            report(ring.error, kErrTimeoutEmpty);
            return false;
        }
        const uint32_t db = uint32_t(n * G::kTileBytes), sb = uint32_t(n * 32);
        mbar_expect_tx(&ring.full[cur.stage], db + sb);
        bulk_g2s(ring.data + size_t(cur.stage) * kStageBytes,
                 run.data + size_t(t) * G::kTileBytes, db, &ring.full[cur.stage]);
        bulk_g2s(ring.scales + size_t(cur.stage) * (kStageScaleBytes / 2),
                 run.scales + size_t(t) * 16, sb, &ring.full[cur.stage]);
        cur.template next<STAGES>();
    }
    return true;
}

} // namespace nut
