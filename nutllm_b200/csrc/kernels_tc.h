#pragma once
/* Launchers of the tensor-pipe kernels (fragment-tile layout). */
#include <algorithm>
#include <cstdint>
#include <cuda_runtime.h>

#include "tiles.h"

namespace nut {

/* A quantised matrix in fragment tiles on the device. */
struct TileMatrix {
    TileShape shape;
    uint8_t *data = nullptr;
    uint16_t *scales = nullptr;
};

/* Default bound on any device-side wait (weights, stages, inputs). */
constexpr uint64_t kDefaultWaitNs = 2000000000ull;

cudaError_t launch_qmatvec_tc(const TileMatrix &m, const float *x, float *y,
                              int *error, uint64_t limit_ns, cudaStream_t stream);

/* Prefill GEMM (gemm_tc.cu).  Y[M][N] (row stride ldy, fp32) =
 * A[M][K] B[N][K]^T with fp16 operands (K a multiple of 64, B allocated
 * with N_alloc >= N rows); device-side timeouts land in *error.  With
 * max_splits > 1 the K dimension may be split over up to that many CTAs
 * per output tile (when the tiles alone fill their waves poorly), each
 * adding its partial product atomically: Y then receives Y + A B^T, so the
 * caller zeroes Y first unless it accumulates. */
cudaError_t gemm_f16(const uint16_t *A, int M, const uint16_t *B, int N, int N_alloc, int K,
                     float *Y, int ldy, int *error, uint64_t limit_ns, cudaStream_t stream,
                     bool accumulate = false, int max_splits = 1);
/* The same product with INT4 block-32 weights dequantised inside the
 * pipeline (gemm_q4_kernel): Wq in the packed layout of pack_q4, the
 * values q * scale rounded to fp16 exactly as dequant_tiles_f16 rounds
 * them.  max_splits as for gemm_f16. */
cudaError_t gemm_q4(const uint16_t *A, int M, const uint8_t *Wq, int N, int K, float *Y, int ldy,
                    int *error, uint64_t limit_ns, cudaStream_t stream, bool accumulate = false,
                    int max_splits = 1);
/* Packed INT4 layout: rows per tile and bytes per (tile, 64-wide K block). */
constexpr int kQ4Rows = 64;
constexpr int kQ4StageBytes = kQ4Rows * 32 + kQ4Rows * 2 * 2;
/* Bytes of the packed layout for an N x K weight matrix (K a multiple of
 * 64): per 64-row tile and 64-wide K block, 64 rows of 32 nibble bytes
 * then 64 x 2 fp16 scale bits. */
size_t q4_packed_bytes(int N, int K);
/* Host packing of INT4 rows in the reference storage (data [N][K_src / 2],
 * scales [N][K_src / 32], K_src a multiple of 32) into that layout, zero
 * past K_src and N. */
void pack_q4(const uint8_t *data, const uint16_t *scales, int N, int K_src, int K,
             uint8_t *out);
/* Fragment tiles (any tile order) -> fp16 [row_tiles * 16][blocks * 32]. */
cudaError_t dequant_tiles_f16(const TileMatrix &m, uint16_t *out, cudaStream_t stream);
/* fp32 [M][K] -> fp16 [M][Kp], zero padded, saturating. */
cudaError_t round_f16(const float *x, int M, int K, int Kp, uint16_t *out, cudaStream_t stream);

} // namespace nut
