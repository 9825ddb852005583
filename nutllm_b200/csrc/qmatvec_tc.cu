/* Quantised matvec y = Q x on the tensor pipe (one matrix, fragment-tile
 * layout).  Replaces the reference's matvec_quantized_threaded
 * (src/quant.cpp:262-321) for block-aligned matrices.
 *
 * Grid: one CTA per SM (at most one per row tile); CTA i owns a contiguous
 * range of row tiles, which is one contiguous run of tiles in HBM.  Warp 8
 * streams the run through the shared-memory ring; warps 0-7 convert x to
 * digits once and then multiply every streamed tile pair. */
#include <cstdio>

#include "kernels.h"
#include "kernels_tc.h"
#include "stream.cuh"

namespace nut {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = (kWarps + 1) * 32;

struct QTParams {
    const uint8_t *tiles;
    const uint16_t *scales;
    int row_tiles, nb, rows, K;
    const float *x;
    float *y;
    int *error;
    uint64_t limit_ns;
    int stages;
};

struct Smem {
    uint8_t *data;
    uint16_t *scales;
    int8_t *dig;
    float *fac;
    float *red;
    int *fatal;
    uint64_t *full, *empty;
};

__device__ __forceinline__ Smem carve(uint8_t *base, int stages, int nb) {
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
    s.red = reinterpret_cast<float *>(base + off);
    off += 2 * kRowBatch * kWarps * 16 * 4;
    s.fatal = reinterpret_cast<int *>(base + off);
    off += 16;
    off = (off + 15) & ~size_t(15);
    s.full = reinterpret_cast<uint64_t *>(base + off);
    s.empty = s.full + stages;
    return s;
}

size_t smem_bytes(int stages, int nb) {
    size_t off = size_t(stages) * (kStageBytes + kStageScaleBytes) + size_t(nb) * 136 +
                 2 * kRowBatch * kWarps * 16 * 4 + 16;
    off = (off + 15) & ~size_t(15);
    return off + size_t(stages) * 16;
}

template <int TYPE, int kStages>
__global__ void __launch_bounds__(kThreads, 1) qmatvec_tc_kernel(QTParams p) {
    static_assert(kStages >= 2, "ring needs two stages");
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Smem s = carve(smem, kStages, p.nb);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], kWarps);
        }
        *s.fatal = 0;
        fence_barrier_init();
    }
    __syncthreads();
    Ring ring{s.data, s.scales, s.full, s.empty, kStages, p.limit_ns, p.error, s.fatal};
    const int rt0 = int(int64_t(p.row_tiles) * blockIdx.x / gridDim.x);
    const int rt1 = int(int64_t(p.row_tiles) * (blockIdx.x + 1) / gridDim.x);
    constexpr int TB = TileGeom<TYPE>::kTileBytes;
    const TileRun run{p.tiles + size_t(rt0) * p.nb * TB,
                      p.scales + size_t(rt0) * p.nb * 16, (rt1 - rt0) * p.nb, p.nb};
    if (warp == kWarps) {
        if (lane == 0) {
            Cursor cur;
            produce_run_c<TYPE, kStages>(ring, run, cur);
        }
        return;
    }
    make_digits(p.x, p.K, p.nb, warp, kWarps, s.dig, s.fac,
                TYPE == 1 ? 1.0f / 16.0f : 1.0f);
    named_barrier(1, kWarps * 32);
    RowReduce rr{s.red, 0};
    Cursor cur;
    float *y = p.y;
    const int rows = p.rows;
    /* every block's digits are written before the barrier above: the
     * rotating pair assignment is safe here */
    consume_run<TYPE, kWarps, kStages, true>(ring, run, cur, s.dig, s.fac, rr, warp, 1,
                      [&](int rt, float v) {
                          const int row = (rt0 + rt) * 16 + lane;
                          if (lane < 16 && row < rows)
                              y[row] = v;
                      });
}

int g_sms = 0;
int g_max_smem = 0;

void device_limits() {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&g_max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
}

} // namespace

cudaError_t launch_qmatvec_tc(const TileMatrix &m, const float *x, float *y,
                              int *error, uint64_t limit_ns, cudaStream_t stream) {
    if (g_sms == 0)
        device_limits();
    const int nb = int(m.shape.blocks);
    /* ten stages when the activation digits leave room, else six */
    const int stages = smem_bytes(10, nb) <= size_t(g_max_smem) ? 10 : 6;
    const size_t smem = smem_bytes(stages, nb);
    if (smem > size_t(g_max_smem))
        return cudaErrorInvalidValue;
    QTParams p{m.data, m.scales, int(m.shape.row_tiles), nb, int(m.shape.rows),
               int(m.shape.cols), x, y, error, limit_ns, stages};
    const int grid = int(std::min<int64_t>(g_sms, m.shape.row_tiles));
    auto go = [&](auto kernel) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(smem));
        kernel<<<grid, kThreads, smem, stream>>>(p);
        nut::count_launches(1);
    };
    if (m.shape.type == 1)
        stages == 10 ? go(qmatvec_tc_kernel<1, 10>) : go(qmatvec_tc_kernel<1, 6>);
    else
        stages == 10 ? go(qmatvec_tc_kernel<0, 10>) : go(qmatvec_tc_kernel<0, 6>);
    return cudaGetLastError();
}

} // namespace nut
