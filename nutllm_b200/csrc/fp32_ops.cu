/* fp32 matrix products of the reference's own kernel benches, in the
 * reference build's exact arithmetic order, so results are bit-identical:
 *
 *   matmul_threaded (src/threading.cpp:163-181): C = A B, every output the
 *     k-sequential chain out = fma(a[m][k], b[k][n], out) from +0 (the build
 *     contracts the vectorised update into one fused multiply-add)
 *   matvec_threaded (src/threading.cpp:183-198): y[r] = sum over columns in
 *     order of the rounded products w[r][c] * x[c] (unfused), except that
 *     the build's scalar loop over the last cols % 4 columns (after the
 *     8-wide blocks and one 4-wide block) is contracted into fused
 *     multiply-adds
 *
 * GEMM: 64 x 64 output tile per CTA, 256 threads with 4 x 4 outputs each,
 * A and B tiles of 16 k-steps staged in shared memory; each output's k loop
 * runs in order across tiles.
 * Matvec: one warp per 32 rows.  Column chunks of 32 x 32 stream through a
 * ring of shared-memory stages (cp.async, 16 bytes per copy, kMvStages
 * chunks in flight); lane l adds row l's 32 products of a chunk in column
 * order, so each row is one sequential sum over all columns.
 */
#include <cstdint>
#include <cuda_runtime.h>

#include "kernels.h"

namespace nut {
namespace {

constexpr int kGB = 64, kGK = 16, kGT = 4; /* tile, k-step, outputs per thread side */

__global__ void __launch_bounds__(256)
sgemm_kernel(const float *__restrict__ A, const float *__restrict__ B, float *__restrict__ C,
             int M, int K, int N) {
    __shared__ float As[kGK][kGB + 4];
    __shared__ float Bs[kGK][kGB + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * kGB, n0 = blockIdx.x * kGB;
    float acc[kGT][kGT];
#pragma unroll
    for (int i = 0; i < kGT; i++)
#pragma unroll
        for (int j = 0; j < kGT; j++)
            acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += kGK) {
        /* 64 x 16 of A (transposed into As[k][m]) and 16 x 64 of B */
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int idx = threadIdx.x + r * 256;
            const int am = idx / kGK, ak = idx % kGK;
            const int gm = m0 + am, gk = k0 + ak;
            As[ak][am] = gm < M && gk < K ? A[size_t(gm) * K + gk] : 0.0f;
            const int bk = idx / kGB, bn = idx % kGB;
            const int gk2 = k0 + bk, gn = n0 + bn;
            Bs[bk][bn] = gk2 < K && gn < N ? B[size_t(gk2) * N + gn] : 0.0f;
        }
        __syncthreads();
        const int kn = min(kGK, K - k0); /* no padded k-steps enter the chains */
        for (int kk = 0; kk < kn; kk++) {
            float a[kGT], b[kGT];
#pragma unroll
            for (int i = 0; i < kGT; i++)
                a[i] = As[kk][ty * kGT + i];
#pragma unroll
            for (int j = 0; j < kGT; j++)
                b[j] = Bs[kk][tx * kGT + j];
#pragma unroll
            for (int i = 0; i < kGT; i++)
#pragma unroll
                for (int j = 0; j < kGT; j++)
                    acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < kGT; i++) {
        const int gm = m0 + ty * kGT + i;
        if (gm >= M)
            continue;
#pragma unroll
        for (int j = 0; j < kGT; j++) {
            const int gn = n0 + tx * kGT + j;
            if (gn < N)
                C[size_t(gm) * N + gn] = acc[i][j];
        }
    }
}

/* 36 stages x 4.5 KB of dynamic shared memory: 144 KB of weights in flight
 * per warp (one warp per SM), enough to cover HBM latency, while each row's
 * sequential sum (the order the reference fixes) runs alongside. */
constexpr int kMvStages = 36;
constexpr int kMvStage = 32 * 36 + 32; /* floats: 32 x 32 weights (padded rows) + x chunk */
constexpr size_t kMvSmem = size_t(kMvStages) * kMvStage * 4;

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

/* One warp per 32 rows; cols a multiple of 32, W and x 16-byte aligned
 * (the fast path); other shapes use matvec_rows_kernel below. */
__global__ void __launch_bounds__(32)
matvec_chunks_kernel(const float *__restrict__ W, const float *__restrict__ x,
                     float *__restrict__ y, int rows, int cols) {
    extern __shared__ __align__(16) float mv_smem[];
    const int lane = threadIdx.x, r0 = blockIdx.x * 32;
    const int chunks = cols / 32;
    auto stage = [&](int c) { return mv_smem + size_t(c % kMvStages) * kMvStage; };
    auto issue = [&](int c) {
        float(*tile)[36] = reinterpret_cast<float(*)[36]>(stage(c));
        /* 32 rows x 8 float4 = 256 copies, 8 per lane, plus the x chunk */
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int idx = lane + i * 32, r = idx / 8, q = idx % 8;
            const int gr = min(r0 + r, rows - 1);
            cp_async16(&tile[r][4 * q], W + size_t(gr) * cols + size_t(c) * 32 + 4 * q);
        }
        if (lane < 8)
            cp_async16(stage(c) + 32 * 36 + 4 * lane, x + size_t(c) * 32 + 4 * lane);
    };
    for (int c = 0; c < kMvStages - 1; c++) {
        if (c < chunks)
            issue(c);
        cp_async_commit();
    }
    float sum = 0.0f;
    for (int c = 0; c < chunks; c++) {
        if (c + kMvStages - 1 < chunks)
            issue(c + kMvStages - 1);
        cp_async_commit();
        cp_async_wait<kMvStages - 1>();
        __syncwarp();
        const float(*tile)[36] = reinterpret_cast<const float(*)[36]>(stage(c));
        const float *xs = stage(c) + 32 * 36;
#pragma unroll 8
        for (int k = 0; k < 32; k++)
            sum = __fadd_rn(sum, __fmul_rn(tile[lane][k], xs[k]));
        __syncwarp();
    }
    cp_async_wait<0>();
    if (r0 + lane < rows)
        y[r0 + lane] = sum;
}

/* Any shape: one thread per row, sequential over the columns (the fused
 * tail as in the reference build). */
__global__ void matvec_rows_kernel(const float *__restrict__ W, const float *__restrict__ x,
                                   float *__restrict__ y, int rows, int cols) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows)
        return;
    const float *w = W + size_t(r) * cols;
    const int rem = cols % 8, unfused = cols - rem + (rem >= 4 ? 4 : 0);
    float sum = 0.0f;
    int c = 0;
    for (; c < unfused; c++)
        sum = __fadd_rn(sum, __fmul_rn(w[c], x[c]));
    for (; c < cols; c++)
        sum = fmaf(w[c], x[c], sum);
    y[r] = sum;
}

} // namespace

cudaError_t matmul_f32(const float *A, const float *B, float *C, int M, int K, int N,
                       cudaStream_t s) {
    const dim3 grid((N + kGB - 1) / kGB, (M + kGB - 1) / kGB);
    sgemm_kernel<<<grid, 256, 0, s>>>(A, B, C, M, K, N);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t matvec_f32(const float *W, const float *x, float *y, int rows, int cols,
                       cudaStream_t s) {
    const bool fast = cols % 32 == 0 && (reinterpret_cast<uintptr_t>(W) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (fast) {
        const cudaError_t e = cudaFuncSetAttribute(
            matvec_chunks_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMvSmem));
        if (e != cudaSuccess)
            return e;
        matvec_chunks_kernel<<<(rows + 31) / 32, 32, kMvSmem, s>>>(W, x, y, rows, cols);
    }
    else
        matvec_rows_kernel<<<(rows + 127) / 128, 128, 0, s>>>(W, x, y, rows, cols);
    count_launches(1);
    return cudaGetLastError();
}

} // namespace nut

/* ---- fp32-weight decode helpers ------------------------------------- */

namespace nut {
namespace {

/* out = x * (1 / sqrt(mean(x^2) + eps)) * w, one CTA (src/ops.cpp:111-134;
 * the sum of squares is reduced in a different order than the reference's
 * eight lanes, within the parity tolerance). */
__global__ void rmsnorm_vec_kernel(const float *x, const float *w, float *out, int n) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        ss = fmaf(x[k], x[k], ss);
    for (int o = 16; o > 0; o >>= 1)
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
    for (int i = 0; i < int(blockDim.x >> 5); i++)
        total += red[i];
    const float scale = 1.0f / sqrtf(total / float(n) + 1e-5f);
    for (int k = threadIdx.x; k < n; k += blockDim.x)
        out[k] = x[k] * scale * w[k];
}

__global__ void add_vec_kernel(float *h, const float *y, int n) {
    const int k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < n)
        h[k] += y[k];
}

} // namespace

cudaError_t rmsnorm_vec(const float *x, const float *w, float *out, int n, cudaStream_t s) {
    rmsnorm_vec_kernel<<<1, 1024, 0, s>>>(x, w, out, n);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t add_vec(float *h, const float *y, int n, cudaStream_t s) {
    add_vec_kernel<<<(n + 255) / 256, 256, 0, s>>>(h, y, n);
    count_launches(1);
    return cudaGetLastError();
}

} // namespace nut
