/* Quantised matvec y = Q x on the tensor pipe (one matrix, fragment-tile
 * layout).  Replaces the reference's matvec_quantized_threaded
 * (src/quant.cpp:262-321) for block-aligned matrices.
 *
 * Grid: one CTA per SM (at most one per row tile); CTA i owns a contiguous
 * range of row tiles, which is one contiguous run of tiles in HBM.  The
 * last warp streams the run through a ring of 16 KB shared-memory stages
 * with bulk copies (tiles and their fp16 scales, completion on an
 * mbarrier), after a bulk copy of x itself, which must not queue behind
 * the weights.  The consumer warps turn x into exact integer digits once
 * (stream.cuh); then two groups of 8 warps take alternate stages, so one
 * group's per-stage tail (folding, release of the stage) overlaps the
 * other's products, and within a stage warp w of a group multiplies pairs
 * w, w + 8, ... with two chained s8 mma.sync per pair, independent
 * accumulators per unrolled pair.  There is no barrier inside the stream: a warp folds its
 * pairs into a running sum per row tile, in tile order, and parks each row
 * tile's sum in its own slot part[warp][row] of shared memory; after the
 * last stage one barrier, then y[row] = sum over warps in warp order.  The
 * summation order is therefore fixed (results are bit-reproducible). */
#include <cstdio>

#include "kernels.h"
#include "kernels_tc.h"
#include "stream.cuh"

namespace nut {
namespace {

/* kGroups groups of kGroupWarps consumer warps: group q consumes stages
 * q, q + kGroups, ... */
constexpr int kGroupWarps = 8;
constexpr int kGroups = 2;
constexpr int kWarps = kGroupWarps * kGroups; /* consumer warps */
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kMaxStages = 12;

struct QTParams {
    const uint8_t *tiles;
    const uint16_t *scales;
    int row_tiles, nb, rows, K;
    const float *x;
    float *y;
    int *error;
    uint64_t limit_ns;
    int rows_cta; /* 16 x the most row tiles any CTA owns */
    int stage_x;  /* x is bulk-copied into shared memory ahead of the weights */
};

struct Smem {
    uint8_t *data;
    uint16_t *scales;
    int8_t *dig;
    float *fac;
    float *part; /* [kWarps][rows_cta] */
    uint2 *dl;   /* [nb / 2][32] lane-ordered digits of each block pair */
    float *fl;   /* [nb / 2][32] the lane's activation factor of each pair */
    float *xs;   /* [K] when stage_x */
    int *fatal;
    uint64_t *full, *empty, *xbar;
};

__device__ __forceinline__ Smem carve(uint8_t *base, int stages, int nb, int rows_cta,
                                      int xs_floats) {
    Smem s;
    size_t off = 0;
    s.data = base + off;
    off += size_t(stages) * kStageBytes;
    s.scales = reinterpret_cast<uint16_t *>(base + off);
    off += size_t(stages) * kStageScaleBytes;
    s.dig = reinterpret_cast<int8_t *>(base + off);
    off += size_t(nb) * 128;
    s.fac = reinterpret_cast<float *>(base + off);
    off += size_t(nb) * 8;
    s.part = reinterpret_cast<float *>(base + off);
    off += size_t(kWarps) * rows_cta * 4;
    s.dl = reinterpret_cast<uint2 *>(base + off);
    off += size_t(nb / 2) * 32 * 8;
    s.fl = reinterpret_cast<float *>(base + off);
    off += size_t(nb / 2) * 32 * 4;
    s.xs = reinterpret_cast<float *>(base + off);
    off += size_t(xs_floats) * 4;
    s.fatal = reinterpret_cast<int *>(base + off);
    off += 16;
    off = (off + 15) & ~size_t(15);
    s.full = reinterpret_cast<uint64_t *>(base + off);
    s.empty = s.full + stages;
    s.xbar = s.empty + stages;
    return s;
}

/* Mirrors carve(); every region stays 16-byte aligned (nb is even, rows_cta
 * a multiple of 16 and xs_floats of 4). */
size_t smem_bytes(int stages, int nb, int rows_cta, int xs_floats) {
    size_t off = size_t(stages) * (kStageBytes + kStageScaleBytes) + size_t(nb) * 136 +
                 size_t(kWarps) * rows_cta * 4 + size_t(nb / 2) * 32 * 12 +
                 size_t(xs_floats) * 4 + 16;
    off = (off + 15) & ~size_t(15);
    return off + size_t(stages) * 16 + 16;
}

/* One pair of tiles (row tile rt, blocks b0, b0 + 1): the lane's partial
 * sums for rows g and g + 8, with the two products chained so every lane
 * reads its two digit sums from one accumulator (columns 0-3 carry block
 * b0's digits through the first product only, 4-7 block b0 + 1's through
 * the second). */
template <int TYPE>
__device__ __forceinline__ void pair_sum(const uint8_t *sd, const uint16_t *ss, int tile,
                                         int b0, const uint2 *dl, const float *fl,
                                         float &yg, float &yg8) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    uint32_t a0[4], a1[4];
    load_a<TYPE>(sd, tile, a0);
    load_a<TYPE>(sd, tile + 1, a1);
    const int half = c >> 1;
    const uint2 dg = dl[(b0 >> 1) * 32 + lane];
    const uint32_t bx0 = dg.x, bx1 = dg.y;
    const uint32_t m = g < 4 ? 0xffffffffu : 0u;
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
    const float F = fl[(b0 >> 1) * 32 + lane];
    const uint16_t *sc = ss + (tile + half) * 16;
    yg = tg * (half_bits_to_float(sc[g]) * F);
    yg8 = tg8 * (half_bits_to_float(sc[g + 8]) * F);
}

/* Adds the warp's sum for row tile rt (lanes c of each row group hold
 * parts) into its slots part[warp][16 rt ..]. */
__device__ __forceinline__ void park(float *part_w, int rt, float y, float y8) {
    const int lane = threadIdx.x & 31;
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
    y += __shfl_xor_sync(0xffffffffu, y, 2);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
    if ((lane & 3) == 0) {
        part_w[16 * rt + (lane >> 2)] += y;
        part_w[16 * rt + (lane >> 2) + 8] += y8;
    }
}

/* Digits of every block of x (make_digits' result), with each warp's
 * loads issued in batches of 8 blocks before any is used: one L2 round
 * trip per batch instead of one per block. */
template <bool SHARED>
__device__ void digits_batched(const float *x, int K, int nb, int w, int8_t *dig, float *fac,
                               float a_unit_inv) {
    constexpr int kBatch = 8;
    const int lane = threadIdx.x & 31;
    for (int b0 = w; b0 < nb; b0 += kBatch * kWarps) {
        float v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            const int b = b0 + j * kWarps, k = b * 32 + lane;
            v[j] = b < nb && k < K ? (SHARED ? x[k] : __ldg(x + k)) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++) {
            const int b = b0 + j * kWarps;
            if (b < nb)
                digit_from(v[j], __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v[j]))),
                           b, dig, fac, a_unit_inv);
        }
    }
}

template <int TYPE, int kStages>
__global__ void __launch_bounds__(kThreads, 1) qmatvec_ring_kernel(QTParams p) {
    static_assert(kStages >= 2, "ring needs two stages");
    using G = TileGeom<TYPE>;
    constexpr int PP = G::kChunkTiles / 2 / kGroupWarps; /* pairs per warp per stage */
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Smem s = carve(smem, kStages, p.nb, p.rows_cta, p.stage_x ? p.K : 0);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kGroupWarps);
        }
        mbar_init(s.xbar, 1);
        *s.fatal = 0;
        fence_barrier_init();
    }
    for (int i = threadIdx.x; i < kWarps * p.rows_cta; i += blockDim.x)
        s.part[i] = 0.0f;
    __syncthreads();
    Ring ring{s.data, s.scales, s.full, s.empty, kStages, p.limit_ns, p.error, s.fatal};
    const int rt0 = int(int64_t(p.row_tiles) * blockIdx.x / gridDim.x);
    const int rt1 = int(int64_t(p.row_tiles) * (blockIdx.x + 1) / gridDim.x);
    constexpr int TB = G::kTileBytes;
    const TileRun run{p.tiles + size_t(rt0) * p.nb * TB,
                      p.scales + size_t(rt0) * p.nb * 16, (rt1 - rt0) * p.nb, p.nb};
    /* launched with programmatic stream serialisation, the next kernel of
     * the stream may start as soon as this one's CTAs leave their SMs;
     * everything it reads before its own griddepcontrol.wait is constant */
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp == kWarps) {
        if (lane == 0) {
            /* x may be the previous kernel's output: wait for that grid
             * (a no-op without a programmatic dependency) before reading
             * it; the weights need no wait */
            asm volatile("griddepcontrol.wait;" ::: "memory");
            /* x first: its few bytes must not queue behind the weights */
            if (p.stage_x) {
                mbar_expect_tx(s.xbar, uint32_t(p.K) * 4u);
                bulk_g2s(s.xs, p.x, uint32_t(p.K) * 4u, s.xbar);
            }
            /* two stages, then the rest once x has landed: a full first
             * wave from every SM would queue x behind it */
            Cursor cur;
            const int head = min(run.tiles, 2 * G::kChunkTiles);
            const TileRun first{run.data, run.scales, head, run.nb};
            const TileRun rest{run.data + size_t(head) * TB, run.scales + size_t(head) * 16,
                               run.tiles - head, run.nb};
            if (produce_run_c<TYPE, kStages>(ring, first, cur) && rest.tiles > 0) {
                if (p.stage_x)
                    mbar_wait(s.xbar, 0, p.limit_ns);
                produce_run_c<TYPE, kStages>(ring, rest, cur);
            }
        }
        return;
    }
    /* the previous grid (x's producer, y's last reader) has completed */
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (p.stage_x) {
        if (!mbar_wait(s.xbar, 0, p.limit_ns)) {
            report(p.error, kErrTimeoutInput);
            *reinterpret_cast<volatile int *>(s.fatal) = 1;
        }
        digits_batched<true>(s.xs, p.K, p.nb, warp, s.dig, s.fac,
                             TYPE == 1 ? 1.0f / 16.0f : 1.0f);
    } else {
        digits_batched<false>(p.x, p.K, p.nb, warp, s.dig, s.fac,
                              TYPE == 1 ? 1.0f / 16.0f : 1.0f);
    }
    named_barrier(1, kWarps * 32);
    /* lane-ordered copies: lane (g, c) of pair P takes digit g % 4 of
     * block 2 P + g / 4 at k = 4c.. and 16 + 4c.., and the factor of
     * block 2 P + c / 2, digit pair c % 2 */
    for (int i = threadIdx.x; i < (p.nb / 2) * 32; i += kWarps * 32) {
        const int P = i >> 5, L = i & 31, g = L >> 2, c = L & 3;
        const int8_t *src = s.dig + (2 * P + (g >> 2)) * 128 + (g & 3) * 32 + 4 * c;
        s.dl[i] = make_uint2(*reinterpret_cast<const uint32_t *>(src),
                             *reinterpret_cast<const uint32_t *>(src + 16));
        s.fl[i] = s.fac[2 * (2 * P + (c >> 1)) + (c & 1)];
    }
    named_barrier(1, kWarps * 32);
    /* floor(tile / nb) by a multiply-high: exact for tile * nb < 2^32 */
    const uint32_t inv_nb = uint32_t((0xffffffffull + uint64_t(p.nb)) / uint64_t(p.nb));
    /* row tiles are whole stages: no stage straddles two row tiles */
    const bool whole_stages = p.nb % G::kChunkTiles == 0;
    float *part_w = s.part + size_t(warp) * p.rows_cta;
    const int group = warp / kGroupWarps, gw = warp % kGroupWarps;
    int cur_rt = -1;
    float run_y = 0.0f, run_y8 = 0.0f;
    bool poisoned = false;
    for (int j = group; j * G::kChunkTiles < run.tiles; j += kGroups) {
        const int t0 = j * G::kChunkTiles;
        const int n = min(G::kChunkTiles, run.tiles - t0);
        Cursor cur;
        cur.stage = j % kStages;
        cur.parity = uint32_t(j / kStages) & 1u;
        if (!poisoned)
            poisoned = *reinterpret_cast<volatile int *>(ring.fatal) != 0;
        if (!poisoned && !mbar_wait(&ring.full[cur.stage], cur.parity, ring.limit_ns)) {
            report(ring.error, kErrTimeoutFull);
            *reinterpret_cast<volatile int *>(ring.fatal) = 1;
            poisoned = true;
        }
        if (!poisoned) {
            const uint8_t *sd = ring.data + size_t(cur.stage) * kStageBytes;
            const uint16_t *ss = ring.scales + size_t(cur.stage) * (kStageScaleBytes / 2);
            float y[PP], y8[PP];
            int rt[PP];
            if (n == G::kChunkTiles && whole_stages) {
                /* a whole stage inside one row tile: its row tile and first
                 * block are stage constants, so every load below is a base
                 * plus an immediate, and without guards the pairs' loads
                 * and products interleave */
                const int r = int(__umulhi(uint32_t(t0), inv_nb));
                const int kb = t0 - r * p.nb;
#pragma unroll
                for (int u = 0; u < PP; u++) {
                    const int tl = 2 * (gw + u * kGroupWarps); /* tile within the stage */
                    rt[u] = r;
                    pair_sum<TYPE>(sd, ss, tl, kb + tl, s.dl, s.fl, y[u], y8[u]);
                }
            } else if (n == G::kChunkTiles) {
#pragma unroll
                for (int u = 0; u < PP; u++) {
                    const int tl = 2 * (gw + u * kGroupWarps); /* tile within the stage */
                    const int tile = t0 + tl;
                    rt[u] = int(__umulhi(uint32_t(tile), inv_nb));
                    pair_sum<TYPE>(sd, ss, tl, tile - rt[u] * p.nb, s.dl, s.fl, y[u], y8[u]);
                }
            } else {
#pragma unroll
                for (int u = 0; u < PP; u++) {
                    const int tl = 2 * (gw + u * kGroupWarps);
                    y[u] = y8[u] = 0.0f;
                    rt[u] = -1;
                    if (tl < n) {
                        const int tile = t0 + tl;
                        rt[u] = int(__umulhi(uint32_t(tile), inv_nb));
                        pair_sum<TYPE>(sd, ss, tl, tile - rt[u] * p.nb, s.dl, s.fl, y[u],
                                       y8[u]);
                    }
                }
            }
            /* fold into the running row-tile sum in tile order (rt is warp
             * uniform) */
#pragma unroll
            for (int u = 0; u < PP; u++) {
                if (rt[u] < 0)
                    continue;
                if (rt[u] != cur_rt) {
                    if (cur_rt >= 0)
                        park(part_w, cur_rt, run_y, run_y8);
                    cur_rt = rt[u];
                    run_y = run_y8 = 0.0f;
                }
                run_y += y[u];
                run_y8 += y8[u];
            }
        }
        __syncwarp();
        if (lane == 0 && !poisoned)
            mbar_arrive(&ring.empty[cur.stage]);
    }
    if (cur_rt >= 0)
        park(part_w, cur_rt, run_y, run_y8);
    named_barrier(1, kWarps * 32);
    if (poisoned)
        return;
    const int nrows = (rt1 - rt0) * 16;
    for (int r = threadIdx.x; r < nrows; r += kWarps * 32) {
        float v = s.part[r];
#pragma unroll
        for (int w = 1; w < kWarps; w++)
            v += s.part[size_t(w) * p.rows_cta + r];
        const int row = rt0 * 16 + r;
        if (row < p.rows)
            p.y[row] = v;
    }
}

int g_sms = 0;
int g_max_smem = 0;

void device_limits() {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&g_max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
}

template <int TYPE, int ST>
void go(const QTParams &p, int grid, size_t smem, cudaStream_t stream) {
    auto kernel = qmatvec_ring_kernel<TYPE, ST>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, p);
    nut::count_launches(1);
}

} // namespace

cudaError_t launch_qmatvec_tc(const TileMatrix &m, const float *x, float *y,
                              int *error, uint64_t limit_ns, cudaStream_t stream) {
    if (g_sms == 0)
        device_limits();
    const int nb = int(m.shape.blocks);
    const int grid = int(std::min<int64_t>(g_sms, m.shape.row_tiles));
    const int rows_cta = int((m.shape.row_tiles + grid - 1) / grid) * 16;
    /* the deepest ring (12, 10, 8, 6, 4 stages) that fits beside the digits
     * and the per-warp row sums */
    /* x rides in shared memory when it is 16-byte aligned and a ring of at
     * least 8 stages still fits beside it */
    int K = int(m.shape.cols);
    int stage_x = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && K % 4 == 0 &&
                  smem_bytes(8, nb, rows_cta, K) <= size_t(g_max_smem);
    int stages = 0;
    for (int st : {kMaxStages, 10, 8, 6, 4})
        if (smem_bytes(st, nb, rows_cta, stage_x ? K : 0) <= size_t(g_max_smem)) {
            stages = st;
            break;
        }
    /* tile indices within a CTA's run stay below 2^32 / nb (exact row-tile
     * division), and every tile index fits an int */
    const uint64_t run_tiles = uint64_t(rows_cta / 16) * uint64_t(nb);
    if (stages == 0 || uint64_t(m.shape.row_tiles) * uint64_t(nb) >= (uint64_t(1) << 31) ||
        run_tiles * uint64_t(nb) >= (uint64_t(1) << 32))
        return cudaErrorInvalidValue;
    const size_t smem = smem_bytes(stages, nb, rows_cta, stage_x ? K : 0);
    QTParams p{m.data, m.scales, int(m.shape.row_tiles), nb, int(m.shape.rows),
               K, x, y, error, limit_ns, rows_cta, stage_x};
#define NUT_QMV_GO(T)                                                                    \
    switch (stages) {                                                                    \
    case 12: go<T, 12>(p, grid, smem, stream); break;                                    \
    case 10: go<T, 10>(p, grid, smem, stream); break;                                    \
    case 8: go<T, 8>(p, grid, smem, stream); break;                                      \
    case 6: go<T, 6>(p, grid, smem, stream); break;                                      \
    default: go<T, 4>(p, grid, smem, stream); break;                                     \
    }
    if (m.shape.type == 1) {
        NUT_QMV_GO(1)
    } else {
        NUT_QMV_GO(0)
    }
#undef NUT_QMV_GO
    return cudaGetLastError();
}

} // namespace nut
