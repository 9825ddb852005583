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

} // namespace nut
