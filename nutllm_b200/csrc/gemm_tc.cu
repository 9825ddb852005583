/* Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
 *
 * Y[M][N] = X[M][K] W[N][K]^T for the quantised linear layers when many
 * tokens are processed at once (prefill_quantized, src/quant_model.cpp:
 * 208-220, feeds every prompt token through the same projections; a batch
 * of M tokens turns the N x K matrix-vector products into one dense
 * contraction).  Operands are fp16: W is the quantised matrix dequantised
 * once (q * scale rounded to fp16) and cached beside the fragment tiles; X
 * is rounded to fp16 per call (saturating at +-65504).  Accumulation is
 * fp32 in tensor memory.
 *
 * One CTA computes one 128 x BN output tile:
 *   warp 4 (one lane)  TMA producer: A tile 128 x 64 and B tile BN x 64
 *                      (fp16, 128-byte swizzle) per stage of a ring
 *   warp 5             allocates BN TMEM columns; one lane issues four
 *                      tcgen05.mma (K = 16 each) per stage and commits
 *                      each stage back to its "empty" barrier
 *   warps 0-3          epilogue: wait for the last commit, tcgen05.ld
 *                      their 32-lane quadrant of the accumulator, store
 *                      fp32 rows of Y
 * Every wait is bounded; a timed-out role records an error and stops, and
 * the producer waits (bounded) for the copies it issued before the CTA
 * frees its tensor memory and exits.
 */
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "kernels_tc.h"
#include "stream.cuh"

namespace nut {
namespace {

constexpr int kBM = 128;  /* UMMA M */
constexpr int kBK = 64;   /* 16-bit elements per 128-byte swizzle row */
constexpr int kEpiWarps = 4;
constexpr int kThreadsG = (kEpiWarps + 2) * 32;

enum : int { kGemmErrFull = 11, kGemmErrEmpty = 12, kGemmErrAccum = 13 };

/* fp32 -> fp16, rounded to nearest, saturating at +-65504 (an outlier
 * beyond fp16 range is clamped rather than turned into infinity). */
__device__ __forceinline__ __half to_half_sat(float v) {
    return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}

/* ---- tcgen05 / TMA wrappers ---- */

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t addr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(addr), "r"(cols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

/* D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulation. */
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
        : "memory");
}

/* Arrives on `bar` once every tcgen05.mma issued so far by this thread has
 * completed. */
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
            smem_u32(bar))
        : "memory");
}

/* 16 consecutive fp32 accumulator columns of this thread's TMEM lane. */
__device__ __forceinline__ void tmem_ld16(uint32_t addr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; j++)
        v[j] = __uint_as_float(r[j]);
}

/* Shared-memory matrix descriptor of a K-major tile with 128-byte rows in
 * the 128-byte swizzle: 8-row core groups 1024 bytes apart (stride byte
 * offset 64 x 16 B), leading byte offset 1 (unused by this mode), version
 * 1, swizzle mode 2.  The tile base must be 1024-byte aligned. */
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= uint64_t((addr >> 4) & 0x3FFFu);
    d |= uint64_t(1) << 16;          /* leading byte offset (16 B units) */
    d |= uint64_t(64) << 32;         /* stride byte offset: 1024 B */
    d |= uint64_t(1) << 46;          /* descriptor version */
    d |= uint64_t(2) << 61;          /* 128-byte swizzle */
    return d;
}

/* Instruction descriptor: dense, fp32 accumulator, fp16 A and B (format
 * code 0), both K-major, shape M x N. */
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                      /* accumulator format F32 */
           | (uint32_t(N >> 3) << 17)     /* N / 8 */
           | (uint32_t(M >> 4) << 24);    /* M / 16 */
}

struct GemmArgs {
    int M, N, K;       /* K a multiple of 64 */
    float *Y;          /* [M][ldy] */
    int ldy;
    int accumulate;    /* Y += A B^T instead of Y = A B^T */
    int *error;
    uint64_t limit_ns;
    int splits;        /* K split over gridDim.z; > 1: Y += A B^T by atomic adds */
};

template <int BN, int STAGES>
struct GemmSmem {
    static constexpr int kA = kBM * kBK * 2;  /* 16 KB */
    static constexpr int kB = BN * kBK * 2;
    static constexpr int kStage = kA + kB;
    static constexpr size_t kBytes = size_t(STAGES) * kStage + 1024 /* align */ + 256;
};

template <int BN, int STAGES, int CTAS_PER_SM = 1>
__global__ void __launch_bounds__(kThreadsG, CTAS_PER_SM)
gemm_f16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const GemmArgs g) {
    using S = GemmSmem<BN, STAGES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * S::kStage);
    uint64_t *empty = full + STAGES;
    uint64_t *accum = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    /* blockIdx.x walks the M tiles fastest, so the CTAs that share one B
     * (weight) tile run together and all but the first read it from L2 */
    const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
    /* this CTA's share of the K blocks (split-K over blockIdx.z) */
    const int kb_total = g.K / kBK;
    const int kb0 = int(blockIdx.z) * kb_total / g.splits;
    const int kb_count = (int(blockIdx.z) + 1) * kb_total / g.splits - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kEpiWarps + 1)
        tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kEpiWarps) {
        /* TMA producer */
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < kb_count; kb++) {
                const int s = kb % STAGES;
                const uint32_t par = uint32_t((kb / STAGES) & 1);
                if (kb >= STAGES &&
                    (*abort_flag || !mbar_wait(&empty[s], par ^ 1u, g.limit_ns))) {
                    atomicCAS(g.error, 0, kGemmErrEmpty);
                    *abort_flag = 1;
                    break;
                }
                uint8_t *a = tiles + s * S::kStage;
                mbar_expect_tx(&full[s], uint32_t(S::kStage));
                tma_load_2d(a, &tmA, (kb0 + kb) * kBK, m0, &full[s]);
                tma_load_2d(a + S::kA, &tmB, (kb0 + kb) * kBK, n0, &full[s]);
                issued = kb + 1;
            }
            /* every issued copy has landed before the CTA can exit */
            for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; kb++)
                mbar_wait(&full[kb % STAGES], uint32_t((kb / STAGES) & 1), g.limit_ns);
        }
    } else if (warp == kEpiWarps + 1) {
        /* MMA issuer */
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kBM, BN);
            for (int kb = 0; kb < kb_count; kb++) {
                const int s = kb % STAGES;
                const uint32_t par = uint32_t((kb / STAGES) & 1);
                if (*abort_flag || !mbar_wait(&full[s], par, g.limit_ns)) {
                    atomicCAS(g.error, 0, kGemmErrFull);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(tiles + s * S::kStage), b = a + S::kA;
#pragma unroll
                for (int k = 0; k < kBK / 16; k++)
                    umma_f16(tmem, smem_desc_sw128(a + k * 32), smem_desc_sw128(b + k * 32),
                              idesc, (kb | k) != 0);
                umma_commit(&empty[s]);
            }
            umma_commit(accum);
        }
        __syncwarp();
    } else {
        /* epilogue: warp w owns TMEM lanes (rows) 32 w .. 32 w + 31 */
        bool ok = mbar_wait(accum, 0u, g.limit_ns);
        if (!ok)
            atomicCAS(g.error, 0, kGemmErrAccum);
        ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
        tc_fence_after();
        const int row = m0 + warp * 32 + lane;
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c), v);
                if (row < g.M && g.splits > 1) {
                    /* split-K: every split adds its partial product */
                    float *y = g.Y + size_t(row) * g.ldy + n0 + c;
                    if (n0 + c + 16 <= g.N && (g.ldy % 4) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            asm volatile(
                                "red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n"
                                ::"l"(y + j), "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]),
                                "f"(v[j + 3])
                                : "memory");
                    } else {
                        for (int j = 0; j < 16; j++)
                            if (n0 + c + j < g.N)
                                atomicAdd(y + j, v[j]);
                    }
                } else if (row < g.M) {
                    float *y = g.Y + size_t(row) * g.ldy + n0 + c;
                    if (n0 + c + 16 <= g.N && (g.ldy % 4) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                            if (g.accumulate) {
                                const float4 r = *reinterpret_cast<const float4 *>(y + j);
                                o.x += r.x, o.y += r.y, o.z += r.z, o.w += r.w;
                            }
                            *reinterpret_cast<float4 *>(y + j) = o;
                        }
                    } else {
                        for (int j = 0; j < 16; j++)
                            if (n0 + c + j < g.N)
                                y[j] = g.accumulate ? y[j] + v[j] : v[j];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kEpiWarps + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

/* ---- persistent form ----------------------------------------------------

   For products of several waves of tiles: one CTA per SM walks the work
   units u = blockIdx.x, blockIdx.x + gridDim.x, ... (unit = output tile x
   K split; M tiles fastest, so the CTAs of one moment share a weight tile
   in L2).  The accumulator is double-buffered in tensor memory (2 x BN
   columns): while warps 0-3 drain unit i's accumulator to Y, warp 5 already
   multiplies unit i + 1 into the other half, and warp 4 keeps streaming
   stages across unit boundaries.  Barriers: full / empty per stage (as in
   gemm_f16_kernel), acc_full[2] (the MMA warp's commit: an accumulator
   is complete) and acc_empty[2] (the 128 epilogue threads: an accumulator
   has been read).  Every wait is bounded; on a timeout a role records the
   error, raises the CTA's abort flag and stops, the producer still waits
   (bounded) for the copies it issued, and the CTA frees its tensor memory. */

struct PersistArgs {
    int tiles_m, tiles_n, splits, units;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreadsG, 1)
gemm_f16_persist(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const GemmArgs g, const PersistArgs pa) {
    using S = GemmSmem<BN, STAGES>;
    static_assert(2 * BN <= 512, "two accumulators in tensor memory");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * S::kStage);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;  /* [2] */
    uint64_t *acc_empty = acc_full + 2;   /* [2] */
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb_total = g.K / kBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], kEpiWarps * 32);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kEpiWarps + 1)
        tmem_alloc(tmem_slot, 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto unit_of = [&](int u, int &m0, int &n0, int &kb0, int &kbn) {
        const int per = pa.tiles_m * pa.tiles_n;
        const int sp = u / per, t = u - sp * per;
        const int tn = t / pa.tiles_m, tm = t - tn * pa.tiles_m;
        m0 = tm * kBM;
        n0 = tn * BN;
        kb0 = sp * kb_total / pa.splits;
        kbn = (sp + 1) * kb_total / pa.splits - kb0;
    };

    if (warp == kEpiWarps) {
        /* TMA producer: one stage sequence across all of this CTA's units */
        if (lane == 0) {
            int issued = 0;
            bool stop = false;
            for (int u = blockIdx.x; u < pa.units && !stop; u += gridDim.x) {
                int m0, n0, kb0, kbn;
                unit_of(u, m0, n0, kb0, kbn);
                for (int kb = 0; kb < kbn; kb++) {
                    const int s = issued % STAGES;
                    const uint32_t par = uint32_t((issued / STAGES) & 1);
                    if (issued >= STAGES &&
                        (*abort_flag || !mbar_wait(&empty[s], par ^ 1u, g.limit_ns))) {
                        atomicCAS(g.error, 0, kGemmErrEmpty);
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    uint8_t *a = tiles + s * S::kStage;
                    mbar_expect_tx(&full[s], uint32_t(S::kStage));
                    tma_load_2d(a, &tmA, (kb0 + kb) * kBK, m0, &full[s]);
                    tma_load_2d(a + S::kA, &tmB, (kb0 + kb) * kBK, n0, &full[s]);
                    issued++;
                }
            }
            /* every issued copy has landed before the CTA can exit */
            for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; i++)
                mbar_wait(&full[i % STAGES], uint32_t((i / STAGES) & 1), g.limit_ns);
        }
    } else if (warp == kEpiWarps + 1) {
        /* MMA issuer */
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kBM, BN);
            int consumed = 0, local = 0;
            bool stop = false;
            for (int u = blockIdx.x; u < pa.units && !stop; u += gridDim.x, local++) {
                int m0, n0, kb0, kbn;
                unit_of(u, m0, n0, kb0, kbn);
                const int acc = local & 1;
                /* the epilogue has read this accumulator's previous unit */
                if (local >= 2 && (*abort_flag ||
                                   !mbar_wait(&acc_empty[acc], uint32_t(((local >> 1) - 1) & 1),
                                              g.limit_ns))) {
                    atomicCAS(g.error, 0, kGemmErrAccum);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * BN);
                for (int kb = 0; kb < kbn; kb++) {
                    const int s = consumed % STAGES;
                    const uint32_t par = uint32_t((consumed / STAGES) & 1);
                    if (*abort_flag || !mbar_wait(&full[s], par, g.limit_ns)) {
                        atomicCAS(g.error, 0, kGemmErrFull);
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(tiles + s * S::kStage), b = a + S::kA;
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        umma_f16(d, smem_desc_sw128(a + k * 32), smem_desc_sw128(b + k * 32),
                                  idesc, (kb | k) != 0);
                    umma_commit(&empty[s]);
                    consumed++;
                }
                if (!stop)
                    umma_commit(&acc_full[acc]);
            }
        }
        __syncwarp();
    } else {
        /* epilogue: warp w owns TMEM lanes (rows) 32 w .. 32 w + 31 */
        int local = 0;
        for (int u = blockIdx.x; u < pa.units; u += gridDim.x, local++) {
            int m0, n0, kb0, kbn;
            unit_of(u, m0, n0, kb0, kbn);
            const int acc = local & 1;
            bool ok = !*abort_flag &&
                      mbar_wait(&acc_full[acc], uint32_t((local >> 1) & 1), g.limit_ns);
            if (!ok)
                atomicCAS(g.error, 0, kGemmErrAccum);
            ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
            if (!ok) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int row = m0 + warp * 32 + lane;
            const uint32_t base = tmem + (uint32_t(warp * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tmem_ld16(base + uint32_t(c), v);
                if (row >= g.M)
                    continue;
                float *y = g.Y + size_t(row) * g.ldy + n0 + c;
                const bool vec = n0 + c + 16 <= g.N && (g.ldy % 4) == 0;
                if (pa.splits > 1) {
                    if (vec) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            asm volatile(
                                "red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n"
                                ::"l"(y + j), "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]),
                                "f"(v[j + 3])
                                : "memory");
                    } else {
                        for (int j = 0; j < 16; j++)
                            if (n0 + c + j < g.N)
                                atomicAdd(y + j, v[j]);
                    }
                } else if (vec) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        if (g.accumulate) {
                            const float4 r = *reinterpret_cast<const float4 *>(y + j);
                            o.x += r.x, o.y += r.y, o.z += r.z, o.w += r.w;
                        }
                        *reinterpret_cast<float4 *>(y + j) = o;
                    }
                } else {
                    for (int j = 0; j < 16; j++)
                        if (n0 + c + j < g.N)
                            y[j] = g.accumulate ? y[j] + v[j] : v[j];
                }
            }
            /* this accumulator may be overwritten by the unit after next */
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kEpiWarps + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

/* ---- SM-pair persistent form (tcgen05 cta_group::2) -----------------------

   For the same products as gemm_f16_persist when M covers 256-row tiles:
   the two CTAs of a cluster (an SM pair) compute one 256 x 256 output tile
   per work unit with one 2-SM product.  CTA r of the pair stages rows
   m0 + 128 r .. of A and rows n0 + 128 r .. of B (16 KB each per 64-wide K
   block), so each SM streams half of B: 32 KB of operands per stage for
   128 x 256 x 64 products instead of 48 KB in the one-SM form, a third less
   L2-to-SM traffic per flop.  The leader (rank 0) issues
   tcgen05.mma.cta_group::2 (M = 256, N = 256), which multiplies A halves
   and B halves across the pair and leaves rows m0 + 128 r .. of the tile
   in CTA r's tensor memory (256 fp32 columns, double-buffered: 512).
   Barriers: both CTAs' TMA loads complete on the leader's full[s] (it
   expects both CTAs' bytes); the leader's commit arrives on empty[s] and
   on acc_full[a] of both CTAs (multicast arrive of tcgen05.commit); the
   epilogue threads of both CTAs arrive on the leader's acc_empty[a].
   Only loads of this GPU's own memory, none multicast.  Every wait is
   bounded, and both CTAs meet at one cluster barrier before freeing their
   tensor memory. */

constexpr int kPairBN = 256;                 /* tile columns (B rows) per pair */
constexpr uint32_t kPeerMask = 0xFEFFFFFFu;  /* clears the peer bit: rank 0's copy */

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t ncluster_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
/* Shared::cluster address of the same variable in CTA `rank` of the cluster. */
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(
                     cluster_addr)
                 : "memory");
}
/* 2-SM TMA load into this CTA's shared memory, completing on the barrier
 * at cluster address `bar` (the leader's). */
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int x, int y,
                                                 uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t addr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(addr), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
        : "memory");
}
/* Arrives on the barrier at this offset in both CTAs of the pair once every
 * 2-SM product issued so far by this thread has completed. */
__device__ __forceinline__ void umma_commit_pair(uint64_t *bar) {
    const uint16_t both = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;\n" ::"r"(smem_u32(bar)),
        "h"(both)
        : "memory");
}

template <int STAGES>
struct PairSmem {
    static constexpr int kA = kBM * kBK * 2;      /* 16 KB: this CTA's 128 rows of A */
    static constexpr int kB = 128 * kBK * 2;      /* 16 KB: this CTA's 128 rows of B */
    static constexpr int kStage = kA + kB;
    static constexpr size_t kBytes = size_t(STAGES) * kStage + 1024 /* align */ + 256;
};

template <int STAGES>
__global__ void __launch_bounds__(kThreadsG, 1)
gemm_f16_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const GemmArgs g, const PersistArgs pa) {
    using S = PairSmem<STAGES>;
    constexpr int BN = kPairBN;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * S::kStage);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;  /* [2] */
    uint64_t *acc_empty = acc_full + 2;   /* [2] (the leader's counts both CTAs) */
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int pair = int(cluster_id_x()), pairs = int(ncluster_x());
    const int kb_total = g.K / kBK;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], 2 * kEpiWarps * 32);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kEpiWarps + 1)
        tmem_alloc_pair(tmem_slot, 2 * BN);
    tc_fence_before();
    /* both CTAs' barriers are initialised before either signals the other */
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto unit_of = [&](int u, int &m0, int &n0, int &kb0, int &kbn) {
        const int per = pa.tiles_m * pa.tiles_n;
        const int sp = u / per, t = u - sp * per;
        const int tn = t / pa.tiles_m, tm = t - tn * pa.tiles_m;
        m0 = tm * 2 * kBM;
        n0 = tn * BN;
        kb0 = sp * kb_total / pa.splits;
        kbn = (sp + 1) * kb_total / pa.splits - kb0;
    };

    if (warp == kEpiWarps) {
        /* TMA producer of this CTA's halves (both CTAs) */
        if (lane == 0) {
            int issued = 0;
            bool stop = false;
            for (int u = pair; u < pa.units && !stop; u += pairs) {
                int m0, n0, kb0, kbn;
                unit_of(u, m0, n0, kb0, kbn);
                for (int kb = 0; kb < kbn; kb++) {
                    const int s = issued % STAGES;
                    const uint32_t par = uint32_t((issued / STAGES) & 1);
                    if (issued >= STAGES &&
                        (*abort_flag || !mbar_wait(&empty[s], par ^ 1u, g.limit_ns))) {
                        atomicCAS(g.error, 0, kGemmErrEmpty);
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    uint8_t *a = tiles + s * S::kStage;
                    if (rank == 0)
                        mbar_expect_tx(&full[s], uint32_t(2 * S::kStage));
                    const uint32_t bar = smem_u32(&full[s]) & kPeerMask;
                    tma_load_2d_pair(a, &tmA, (kb0 + kb) * kBK, m0 + int(rank) * kBM, bar);
                    tma_load_2d_pair(a + S::kA, &tmB, (kb0 + kb) * kBK, n0 + int(rank) * 128,
                                     bar);
                    issued++;
                }
            }
            /* the leader's full barriers count both CTAs' copies: every
             * issued copy has landed before the leader exits */
            if (rank == 0)
                for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; i++)
                    mbar_wait(&full[i % STAGES], uint32_t((i / STAGES) & 1), g.limit_ns);
        }
    } else if (warp == kEpiWarps + 1) {
        /* MMA issuer: the leader only */
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_f16(2 * kBM, BN);
            int consumed = 0, local = 0;
            bool stop = false;
            for (int u = pair; u < pa.units && !stop; u += pairs, local++) {
                int m0, n0, kb0, kbn;
                unit_of(u, m0, n0, kb0, kbn);
                const int acc = local & 1;
                /* both CTAs' epilogues have read this accumulator's
                 * previous unit */
                if (local >= 2 && (*abort_flag ||
                                   !mbar_wait(&acc_empty[acc], uint32_t(((local >> 1) - 1) & 1),
                                              g.limit_ns))) {
                    atomicCAS(g.error, 0, kGemmErrAccum);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * BN);
                for (int kb = 0; kb < kbn; kb++) {
                    const int s = consumed % STAGES;
                    const uint32_t par = uint32_t((consumed / STAGES) & 1);
                    if (*abort_flag || !mbar_wait(&full[s], par, g.limit_ns)) {
                        atomicCAS(g.error, 0, kGemmErrFull);
                        *abort_flag = 1;
                        stop = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = smem_u32(tiles + s * S::kStage), b = a + S::kA;
#pragma unroll
                    for (int k = 0; k < kBK / 16; k++)
                        umma_f16_pair(d, smem_desc_sw128(a + k * 32),
                                      smem_desc_sw128(b + k * 32), idesc, (kb | k) != 0);
                    umma_commit_pair(&empty[s]);
                    consumed++;
                }
                if (!stop)
                    umma_commit_pair(&acc_full[acc]);
            }
        }
        __syncwarp();
    } else {
        /* epilogue (both CTAs): warp w owns TMEM lanes 32 w .. 32 w + 31,
         * i.e. rows m0 + 128 rank + 32 w + lane of the unit's tile */
        const uint32_t leader_empty0 = map_rank(smem_u32(&acc_empty[0]), 0);
        const uint32_t leader_empty1 = map_rank(smem_u32(&acc_empty[1]), 0);
        int local = 0;
        for (int u = pair; u < pa.units; u += pairs, local++) {
            int m0, n0, kb0, kbn;
            unit_of(u, m0, n0, kb0, kbn);
            const int acc = local & 1;
            bool ok = !*abort_flag &&
                      mbar_wait(&acc_full[acc], uint32_t((local >> 1) & 1), g.limit_ns);
            if (!ok)
                atomicCAS(g.error, 0, kGemmErrAccum);
            ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
            if (!ok) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int row = m0 + int(rank) * kBM + warp * 32 + lane;
            const uint32_t base = tmem + (uint32_t(warp * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tmem_ld16(base + uint32_t(c), v);
                if (row >= g.M)
                    continue;
                float *y = g.Y + size_t(row) * g.ldy + n0 + c;
                const bool vec = n0 + c + 16 <= g.N && (g.ldy % 4) == 0;
                if (pa.splits > 1) {
                    if (vec) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            asm volatile(
                                "red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n"
                                ::"l"(y + j), "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]),
                                "f"(v[j + 3])
                                : "memory");
                    } else {
                        for (int j = 0; j < 16; j++)
                            if (n0 + c + j < g.N)
                                atomicAdd(y + j, v[j]);
                    }
                } else if (vec) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        if (g.accumulate) {
                            const float4 r = *reinterpret_cast<const float4 *>(y + j);
                            o.x += r.x, o.y += r.y, o.z += r.z, o.w += r.w;
                        }
                        *reinterpret_cast<float4 *>(y + j) = o;
                    }
                } else {
                    for (int j = 0; j < 16; j++)
                        if (n0 + c + j < g.N)
                            y[j] = g.accumulate ? y[j] + v[j] : v[j];
                }
            }
            /* this accumulator may be overwritten by the unit after next */
            tc_fence_before();
            mbar_arrive_cluster(acc ? leader_empty1 : leader_empty0);
        }
    }
    tc_fence_before();
    __syncthreads();
    /* the peer's tensor memory is written by the leader's products and read
     * by the peer's epilogue: free it only when both CTAs are done */
    cluster_sync();
    if (warp == kEpiWarps + 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 2 * BN);
    }
}

/* ---- dequantisation and activation rounding ---- */

/* Fragment tiles (any tile order) -> fp16 [row_tiles * 16][blocks * 32]
 * (q * scale exact in fp32, rounded to nearest fp16).  One thread per
 * (tile, lane). */
template <int TYPE>
__global__ void dequant_tiles_kernel(const uint8_t *tiles, const uint16_t *scales, int row_tiles,
                                     int blocks, int order, __half *out) {
    const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t ntiles = int64_t(row_tiles) * blocks;
    if (gid >= ntiles * 32)
        return;
    const int lane = int(gid & 31);
    const int64_t lt = gid >> 5; /* logical tile: row tile lt / blocks, block lt % blocks */
    const int rt = int(lt / blocks), b = int(lt % blocks);
    const int64_t t = order == kPairColumn   ? (int64_t(b >> 1) * row_tiles + rt) * 2 + (b & 1)
                      : order == kBlockColumn ? int64_t(b) * row_tiles + rt
                                              : lt;
    const int g = lane >> 2, c = lane & 3;
    uint32_t a[4];
    if (TYPE == 0) {
        const uint4 p = *reinterpret_cast<const uint4 *>(tiles + t * 512 + 16 * lane);
        a[0] = p.x, a[1] = p.y, a[2] = p.z, a[3] = p.w;
    } else {
        const uint2 p = *reinterpret_cast<const uint2 *>(tiles + t * 256 + 8 * lane);
        a[0] = (p.x << 4) & 0xF0F0F0F0u, a[1] = p.x & 0xF0F0F0F0u;
        a[2] = (p.y << 4) & 0xF0F0F0F0u, a[3] = p.y & 0xF0F0F0F0u;
    }
    const float unit = TYPE == 1 ? 1.0f / 16.0f : 1.0f;
    const float s0 = half_bits_to_float(scales[t * 16 + g]) * unit;
    const float s1 = half_bits_to_float(scales[t * 16 + g + 8]) * unit;
    const int64_t ld = int64_t(blocks) * 32;
    const int64_t r0 = int64_t(rt) * 16 + g, r1 = r0 + 8;
    const int k0 = b * 32 + 4 * c;
    /* a0: row g, cols 4c..4c+3; a1: row g+8, same; a2: row g, 16+4c..;
       a3: row g+8, 16+4c.. (the m16n8k32 A fragment) */
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int64_t row = (r & 1) ? r1 : r0;
        const float s = (r & 1) ? s1 : s0;
        const int k = k0 + ((r & 2) ? 16 : 0);
        __half *dst = out + row * ld + k;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int q = int(int8_t(uint8_t(a[r] >> (8 * j))));
            dst[j] = to_half_sat(float(q) * s);
        }
    }
}

/* fp32 [M][K] -> fp16 [M][Kp] (columns K..Kp-1 zero). */
__global__ void round_f16_kernel(const float *x, int M, int K, int Kp, __half *out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(M) * Kp)
        return;
    const int64_t m = i / Kp;
    const int k = int(i - m * Kp);
    out[i] = to_half_sat(k < K ? x[m * K + k] : 0.0f);
}

/* ---- host side ---- */

/* cuTensorMapEncodeTiled, resolved through the runtime so the library
 * does not link the driver library (it loads on machines without one). */
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return EncodeTiledFn(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

bool encode_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols_elems,
                int box_rows) {
    const EncodeTiledFn encode = encode_fn();
    if (encode == nullptr)
        return false;
    const cuuint64_t dims[2] = {cuuint64_t(cols_elems), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(cols_elems) * 2};
    const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(
        map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box,
        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

/* ---- INT4 weights dequantised in the pipeline ----------------------

   Y[M][N] (+)= X[M][K] W[N][K]^T with W kept as INT4 block-32 weights in a
   packed layout: for every 64-row tile n and 64-wide K block kb, 64 rows of
   32 bytes (the row's 64 nibbles) then 64 x 2 fp16 scale bits (kQ4Stage
   bytes in all, one contiguous bulk copy).  Each 32-bit word holds 8
   consecutive k in the nibble order k0 k2 k4 k6 k1 k3 k5 k7 (bits 0-3 =
   k0, ..., 28-31 = k7), offset by 8 (q + 8, 0..15), so that
   ((w >> 4j) & 0x000F000F) | 0x64006400 is the half2 (1024 + q_2j + 8,
   1024 + q_2j+1 + 8): one subtraction of 1032 gives the exact pair and one
   half2 multiply by the block scale gives q * scale rounded once to fp16,
   the value dequant_tiles_f16 produces.  Per stage:
     warp 4 (one lane)  TMA load of the fp16 X tile (128 x 64) and a bulk copy
                        of the W stage into a staging area, both completing on
                        the stage's "full" barrier
     warps 0-3          dequantise the staged stage: thread t expands row t/2,
                        quant block t%2 (32 nibbles), to fp16 q * scale (the
                        rounding of dequant_tiles_f16), written in the 128-byte
                        swizzle the MMA descriptor reads; a proxy fence makes
                        the stores visible to the tensor core, then one arrive
                        per warp on the stage's "ready" barrier
     warp 5             waits "full" and "ready", issues the MMAs, commits
                        to "empty"
   and warps 0-3 run the usual epilogue after the last stage. */
constexpr int kQ4N = kQ4Rows;                     /* weight rows per tile */
constexpr int kQ4Bytes = kQ4N * 32;               /* nibbles per stage */
constexpr int kQ4Stage = kQ4StageBytes;           /* + scales */
static_assert(kQ4Stage == kQ4Bytes + kQ4N * 2 * 2, "packed INT4 stage layout");

template <int STAGES>
struct Q4Smem {
    static constexpr int kA = kBM * kBK * 2;  /* 16 KB */
    static constexpr int kB = kQ4N * kBK * 2; /* 8 KB */
    static constexpr int kTile = kA + kB;     /* 1024-byte multiple */
    static constexpr size_t kBytes =
        size_t(STAGES) * (kTile + kQ4Stage) + 1024 /* align */ + 512;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

template <int STAGES, int CTAS_PER_SM = 1>
__global__ void __launch_bounds__(kThreadsG, CTAS_PER_SM)
gemm_q4_kernel(const __grid_constant__ CUtensorMap tmA, const uint8_t *wq, const GemmArgs g) {
    using S = Q4Smem<STAGES>;
    constexpr int BN = kQ4N;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *tiles = smem;                                 /* [STAGES][A | B] */
    uint8_t *staging = smem + STAGES * S::kTile;           /* [STAGES][kQ4Stage] */
    uint64_t *full = reinterpret_cast<uint64_t *>(staging + STAGES * kQ4Stage);
    uint64_t *ready = full + STAGES;
    uint64_t *empty = ready + STAGES;
    uint64_t *accum = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kBM, nt = blockIdx.y, n0 = nt * BN;
    const int kb_total = g.K / kBK;
    const int kb0 = int(blockIdx.z) * kb_total / g.splits;
    const int kb_count = (int(blockIdx.z) + 1) * kb_total / g.splits - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], kEpiWarps);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == kEpiWarps + 1)
        tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kEpiWarps) {
        /* producer */
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < kb_count; kb++) {
                const int s = kb % STAGES;
                const uint32_t par = uint32_t((kb / STAGES) & 1);
                if (kb >= STAGES &&
                    (*abort_flag || !mbar_wait(&empty[s], par ^ 1u, g.limit_ns))) {
                    atomicCAS(g.error, 0, kGemmErrEmpty);
                    *abort_flag = 1;
                    break;
                }
                uint8_t *a = tiles + s * S::kTile;
                mbar_expect_tx(&full[s], uint32_t(S::kA + kQ4Stage));
                tma_load_2d(a, &tmA, (kb0 + kb) * kBK, m0, &full[s]);
                bulk_g2s(staging + s * kQ4Stage,
                         wq + (size_t(nt) * kb_total + size_t(kb0 + kb)) * kQ4Stage,
                         uint32_t(kQ4Stage), &full[s]);
                issued = kb + 1;
            }
            for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; kb++)
                mbar_wait(&full[kb % STAGES], uint32_t((kb / STAGES) & 1), g.limit_ns);
        }
    } else if (warp == kEpiWarps + 1) {
        /* MMA issuer */
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(kBM, BN);
            for (int kb = 0; kb < kb_count; kb++) {
                const int s = kb % STAGES;
                const uint32_t par = uint32_t((kb / STAGES) & 1);
                if (*abort_flag || !mbar_wait(&full[s], par, g.limit_ns) ||
                    !mbar_wait(&ready[s], par, g.limit_ns)) {
                    atomicCAS(g.error, 0, kGemmErrFull);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a = smem_u32(tiles + s * S::kTile), b = a + S::kA;
#pragma unroll
                for (int k = 0; k < kBK / 16; k++)
                    umma_f16(tmem, smem_desc_sw128(a + k * 32), smem_desc_sw128(b + k * 32),
                             idesc, (kb | k) != 0);
                umma_commit(&empty[s]);
            }
            umma_commit(accum);
        }
        __syncwarp();
    } else {
        /* dequantisers: thread t owns row t / 2, quant block t % 2 */
        const int t = threadIdx.x, r = t >> 1, h = t & 1;
        for (int kb = 0; kb < kb_count; kb++) {
            const int s = kb % STAGES;
            const uint32_t par = uint32_t((kb / STAGES) & 1);
            bool ok = !*abort_flag && mbar_wait(&full[s], par, g.limit_ns);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) {
                    atomicCAS(g.error, 0, kGemmErrFull);
                    *abort_flag = 1;
                }
                break;
            }
            const uint8_t *st = staging + s * kQ4Stage;
            const uint4 q = *reinterpret_cast<const uint4 *>(st + r * 32 + h * 16);
            const uint16_t sbits = reinterpret_cast<const uint16_t *>(st + kQ4Bytes)[r * 2 + h];
            const __half2 sc2 = __halves2half2(__ushort_as_half(sbits), __ushort_as_half(sbits));
            const __half2 bias = __halves2half2(__ushort_as_half(0x6408),
                                                __ushort_as_half(0x6408)); /* 1032 */
            uint8_t *brow = tiles + s * S::kTile + S::kA + r * 128;
            const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                /* 8 values k = 32 h + 8 c .. + 7 from one 32-bit word */
                const uint32_t w = words[c];
                uint32_t packed[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t bits = ((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u;
                    const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&bits),
                                                      bias),
                                              sc2);
                    packed[j] = *reinterpret_cast<const uint32_t *>(&v);
                }
                const int chunk = (4 * h + c) ^ (r & 7);
                *reinterpret_cast<uint4 *>(brow + chunk * 16) =
                    make_uint4(packed[0], packed[1], packed[2], packed[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&ready[s]);
        }
        /* epilogue: warp w owns TMEM lanes (rows) 32 w .. 32 w + 31 */
        bool ok = mbar_wait(accum, 0u, g.limit_ns);
        if (!ok)
            atomicCAS(g.error, 0, kGemmErrAccum);
        ok = __all_sync(0xffffffffu, ok) && !*abort_flag;
        tc_fence_after();
        const int row = m0 + warp * 32 + lane;
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 16) {
                float v[16];
                tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c), v);
                if (row >= g.M)
                    continue;
                float *y = g.Y + size_t(row) * g.ldy + n0 + c;
                const bool vec = n0 + c + 16 <= g.N && (g.ldy % 4) == 0;
                if (g.splits > 1 && vec) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        asm volatile(
                            "red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n"
                            ::"l"(y + j), "f"(v[j]), "f"(v[j + 1]), "f"(v[j + 2]),
                            "f"(v[j + 3])
                            : "memory");
                } else if (g.splits > 1) {
                    for (int j = 0; j < 16; j++)
                        if (n0 + c + j < g.N)
                            atomicAdd(y + j, v[j]);
                } else if (vec) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        if (g.accumulate) {
                            const float4 p = *reinterpret_cast<const float4 *>(y + j);
                            o.x += p.x, o.y += p.y, o.z += p.z, o.w += p.w;
                        }
                        *reinterpret_cast<float4 *>(y + j) = o;
                    }
                } else {
                    for (int j = 0; j < 16; j++)
                        if (n0 + c + j < g.N)
                            y[j] = g.accumulate ? y[j] + v[j] : v[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kEpiWarps + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, BN);
    }
}

template <int BN, int STAGES, int CTAS_PER_SM = 1>
cudaError_t launch_bn(const CUtensorMap &a, const CUtensorMap &b, const GemmArgs &g,
                      cudaStream_t stream) {
    using S = GemmSmem<BN, STAGES>;
    static_assert(CTAS_PER_SM * (S::kBytes + 1024) <= 228 * 1024, "shared memory per SM");
    auto k = gemm_f16_kernel<BN, STAGES, CTAS_PER_SM>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::kBytes));
    if (e != cudaSuccess)
        return e;
    const dim3 grid((g.M + kBM - 1) / kBM, (g.N + BN - 1) / BN, g.splits);
    k<<<grid, kThreadsG, S::kBytes, stream>>>(a, b, g);
    count_launches(1);
    return cudaGetLastError();
}

template <int BN, int STAGES>
cudaError_t launch_persist(const CUtensorMap &a, const CUtensorMap &b, const GemmArgs &g,
                           const PersistArgs &pa, int grid, cudaStream_t stream) {
    using S = GemmSmem<BN, STAGES>;
    static_assert(S::kBytes + 64 <= 227 * 1024, "shared memory per CTA");
    auto k = gemm_f16_persist<BN, STAGES>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::kBytes));
    if (e != cudaSuccess)
        return e;
    k<<<grid, kThreadsG, S::kBytes, stream>>>(a, b, g, pa);
    count_launches(1);
    return cudaGetLastError();
}

/* Launches the SM-pair kernel with as many pairs as fit at once (at most
 * one per work unit).  cudaErrorNotSupported when no pair fits. */
template <int STAGES>
cudaError_t launch_pair(const CUtensorMap &a, const CUtensorMap &b, const GemmArgs &g,
                        const PersistArgs &pa, cudaStream_t stream) {
    using S = PairSmem<STAGES>;
    static_assert(S::kBytes + 64 <= 227 * 1024, "shared memory per CTA");
    auto k = gemm_f16_pair<STAGES>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::kBytes));
    if (e != cudaSuccess)
        return e;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kThreadsG);
    cfg.dynamicSmemBytes = S::kBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int fits = -1; /* pairs resident at once (same for every call) */
    if (fits < 0) {
        cfg.gridDim = dim3(2 * 74);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k, &cfg) != cudaSuccess)
            n = 0;
        fits = n;
    }
    if (fits <= 0)
        return cudaErrorNotSupported;
    cfg.gridDim = dim3(2 * std::min(fits, pa.units));
    e = cudaLaunchKernelEx(&cfg, k, a, b, g, pa);
    count_launches(1);
    return e != cudaSuccess ? e : cudaGetLastError();
}

template <int STAGES, int CTAS_PER_SM = 1>
cudaError_t launch_q4(const CUtensorMap &a, const uint8_t *wq, const GemmArgs &g,
                      cudaStream_t stream) {
    using S = Q4Smem<STAGES>;
    static_assert(CTAS_PER_SM * (S::kBytes + 1024) <= 228 * 1024, "shared memory per SM");
    auto k = gemm_q4_kernel<STAGES, CTAS_PER_SM>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(S::kBytes));
    if (e != cudaSuccess)
        return e;
    const dim3 grid((g.M + kBM - 1) / kBM, (g.N + kQ4N - 1) / kQ4N, g.splits);
    k<<<grid, kThreadsG, S::kBytes, stream>>>(a, wq, g);
    count_launches(1);
    return cudaGetLastError();
}

/* CTAs per SM for the 64- and 128-column tiles: 2 (measured on B200,
 * Llama-2-7B-shape batch-64 decode step: 58.7k -> 68.7k tok/s; 3 and 4
 * were no better), or 1 with NUTLLM_GEMM_CTAS_PER_SM=1 (read once). */
int ctas_per_sm() {
    static const int n = [] {
        const char *v = std::getenv("NUTLLM_GEMM_CTAS_PER_SM");
        return v != nullptr && std::atoi(v) == 1 ? 1 : 2;
    }();
    return n;
}

} // namespace

cudaError_t dequant_tiles_f16(const TileMatrix &m, uint16_t *out, cudaStream_t stream) {
    const int64_t threads = int64_t(m.shape.row_tiles) * m.shape.blocks * 32;
    const int grid = int((threads + 255) / 256);
    auto *o = reinterpret_cast<__half *>(out);
    const int rt = int(m.shape.row_tiles), nb = int(m.shape.blocks), order = m.shape.order;
    if (m.shape.type == 1)
        dequant_tiles_kernel<1><<<grid, 256, 0, stream>>>(m.data, m.scales, rt, nb, order, o);
    else
        dequant_tiles_kernel<0><<<grid, 256, 0, stream>>>(m.data, m.scales, rt, nb, order, o);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t round_f16(const float *x, int M, int K, int Kp, uint16_t *out, cudaStream_t stream) {
    const int64_t n = int64_t(M) * Kp;
    round_f16_kernel<<<int((n + 255) / 256), 256, 0, stream>>>(
        x, M, K, Kp, reinterpret_cast<__half *>(out));
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t gemm_f16(const uint16_t *A, int M, const uint16_t *B, int N, int N_alloc, int K,
                      float *Y, int ldy, int *error, uint64_t limit_ns, cudaStream_t stream,
                      bool accumulate, int max_splits) {
    if (M <= 0 || N <= 0 || K <= 0 || K % kBK != 0 ||
        (reinterpret_cast<uintptr_t>(A) & 15) != 0 || (reinterpret_cast<uintptr_t>(B) & 15) != 0)
        return cudaErrorInvalidValue;
    /* the widest output tile (256, 128, 64 columns) that still gives every
     * SM a tile, so small matrices do not leave most of the GPU idle */
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int mt = (M + kBM - 1) / kBM;
    int bn = 256;
    while (bn > 64 && mt * ((N + bn - 1) / bn) < sms)
        bn /= 2;
    /* Tiles of 64 or 128 columns run several CTAs per SM with fewer stages
     * each (about the same bytes in flight per SM): while one CTA fills its
     * ring or drains its accumulator, the others stream. */
    const int per_sm = bn <= 128 ? ctas_per_sm() : 1;
    const int slots = sms * per_sm;
    /* split K (at least 4 K blocks per split) so that the CTAs fill their
     * waves best: a grid of t CTAs runs ceil(t / slots) waves; the fewest
     * splits within 2 % of the best fill win (each split adds its partial
     * product atomically) */
    int splits = 1;
    const int tiles = mt * ((N + bn - 1) / bn), kbs = K / kBK;
    double best = 0.0;
    for (int sp = 1; sp <= max_splits && kbs / sp >= 4; sp++) {
        const int t = tiles * sp, waves = (t + slots - 1) / slots;
        const double fill = double(t) / double(waves * slots);
        if (fill > best + 0.02) {
            best = fill;
            splits = sp;
        }
    }
    CUtensorMap ma, mb;
    if (!encode_map(&ma, A, M, K, kBM) || !encode_map(&mb, B, N_alloc, K, bn))
        return cudaErrorInvalidValue;
    /* several waves of 256-column tiles: one persistent CTA per SM, the
     * accumulator double-buffered in tensor memory so each unit's epilogue
     * overlaps the next unit's products (NUTLLM_GEMM_PERSIST=0: one CTA per
     * unit, as below) */
    static const bool persist_on = [] {
        const char *e = std::getenv("NUTLLM_GEMM_PERSIST");
        return e == nullptr || std::atoi(e) != 0;
    }();
    /* SM pairs (two 128-row halves of a 256 x 256 tile per cluster) when M
     * spans more than one 128-row tile (NUTLLM_GEMM_PAIR=0: one SM per tile) */
    static const bool pair_on = [] {
        const char *e = std::getenv("NUTLLM_GEMM_PAIR");
        return e == nullptr || std::atoi(e) != 0;
    }();
    if (persist_on && pair_on && bn == 256 && tiles * splits > slots && M > kBM) {
        /* no split K: these products already span several waves of pairs,
         * and a split's atomic epilogue costs more than the wave it fills
         * (32000 x 2048 x 512: 76 us unsplit, 113 us in two splits) */
        const int mt2 = (M + 2 * kBM - 1) / (2 * kBM), nt2 = (N + 255) / 256;
        CUtensorMap mb2;
        if (!encode_map(&mb2, B, N_alloc, K, 128))
            return cudaErrorInvalidValue;
        const GemmArgs g{M, N, K, Y, ldy, accumulate ? 1 : 0, error, limit_ns, 1};
        const PersistArgs pa{mt2, nt2, 1, mt2 * nt2};
        const cudaError_t e = launch_pair<6>(ma, mb2, g, pa, stream);
        if (e != cudaErrorNotSupported)
            return e;
    }
    if (persist_on && bn == 256 && tiles * splits > slots) {
        const GemmArgs g{M, N, K, Y, ldy, accumulate ? 1 : 0, error, limit_ns, splits};
        const PersistArgs pa{mt, (N + bn - 1) / bn, splits, tiles * splits};
        return launch_persist<256, 4>(ma, mb, g, pa, std::min(sms, pa.units), stream);
    }
    const GemmArgs g{M, N, K, Y, ldy, accumulate ? 1 : 0, error, limit_ns, splits};
    if (bn == 256)
        return launch_bn<256, 4>(ma, mb, g, stream);
    if (bn == 128)
        return per_sm == 2 ? launch_bn<128, 3, 2>(ma, mb, g, stream)
                           : launch_bn<128, 6>(ma, mb, g, stream);
    return per_sm == 2 ? launch_bn<64, 4, 2>(ma, mb, g, stream)
                       : launch_bn<64, 8>(ma, mb, g, stream);
}

size_t q4_packed_bytes(int N, int K) {
    return size_t((N + kQ4N - 1) / kQ4N) * size_t(K / kBK) * size_t(kQ4Stage);
}

void pack_q4(const uint8_t *data, const uint16_t *scales, int N, int K_src, int K,
             uint8_t *out) {
    const int tiles = (N + kQ4N - 1) / kQ4N, kbs = K / kBK;
    for (int nt = 0; nt < tiles; nt++)
        for (int kb = 0; kb < kbs; kb++) {
            uint8_t *st = out + (size_t(nt) * kbs + kb) * kQ4Stage;
            uint16_t *ss = reinterpret_cast<uint16_t *>(st + kQ4Bytes);
            for (int r = 0; r < kQ4N; r++) {
                const int row = nt * kQ4N + r;
                for (int h = 0; h < 2; h++) {
                    const int blk = kb * 2 + h; /* quant block within the row */
                    const bool in = row < N && (blk + 1) * 32 <= K_src;
                    uint8_t *dst = st + r * 32 + h * 16;
                    if (in) {
                        /* reference order: element k in byte k / 2, even k in
                         * the low nibble; packed: per word of 8 values the
                         * order k0 k2 k4 k6 k1 k3 k5 k7, offset by 8 */
                        const uint8_t *src = data + size_t(row) * (K_src / 2) + blk * 16;
                        for (int wd = 0; wd < 4; wd++) {
                            uint32_t word = 0;
                            for (int k = 0; k < 8; k++) {
                                const uint8_t byte = src[wd * 4 + k / 2];
                                const uint32_t nib = ((k & 1) ? byte >> 4 : byte) & 0xFu;
                                const uint32_t off = (nib ^ 8u) & 0xFu; /* q + 8 */
                                const int slot = (k & 1) ? 4 + k / 2 : k / 2;
                                word |= off << (4 * slot);
                            }
                            for (int i = 0; i < 4; i++)
                                dst[wd * 4 + i] = uint8_t(word >> (8 * i));
                        }
                        ss[r * 2 + h] = scales[size_t(row) * (K_src / 32) + blk];
                    } else {
                        /* q = 0 (offset 8) with a zero scale */
                        for (int i = 0; i < 16; i++)
                            dst[i] = 0x88;
                        ss[r * 2 + h] = 0;
                    }
                }
            }
        }
}

cudaError_t gemm_q4(const uint16_t *A, int M, const uint8_t *Wq, int N, int K, float *Y, int ldy,
                    int *error, uint64_t limit_ns, cudaStream_t stream, bool accumulate,
                    int max_splits) {
    if (M <= 0 || N <= 0 || K <= 0 || K % kBK != 0 ||
        (reinterpret_cast<uintptr_t>(A) & 15) != 0 || (reinterpret_cast<uintptr_t>(Wq) & 15) != 0)
        return cudaErrorInvalidValue;
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int mt = (M + kBM - 1) / kBM;
    const int per_sm = ctas_per_sm(), slots = sms * per_sm;
    int splits = 1;
    const int tiles = mt * ((N + kQ4N - 1) / kQ4N), kbs = K / kBK;
    double best = 0.0;
    for (int sp = 1; sp <= max_splits && kbs / sp >= 4; sp++) {
        const int t = tiles * sp, waves = (t + slots - 1) / slots;
        const double fill = double(t) / double(waves * slots);
        if (fill > best + 0.02) {
            best = fill;
            splits = sp;
        }
    }
    CUtensorMap ma;
    if (!encode_map(&ma, A, M, K, kBM))
        return cudaErrorInvalidValue;
    const GemmArgs g{M, N, K, Y, ldy, accumulate ? 1 : 0, error, limit_ns, splits};
    return per_sm == 2 ? launch_q4<4, 2>(ma, Wq, g, stream) : launch_q4<8>(ma, Wq, g, stream);
}

} // namespace nut
