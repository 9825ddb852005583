/* Greedy head that allocates nothing: nut_greedy_head_static.
 *
 * For callers that cannot call cudaMalloc or cudaFree — a host runtime
 * that hands this library memory from its own arena, or code that issues
 * work while allocation is not allowed — and so cannot create the model
 * and KV-cache objects whose buffers the rest of the C ABI owns.  The
 * caller passes every input and output as device memory; the only scratch
 * the kernels need (one 64-bit argmax accumulator per batch row) lives in
 * a fixed array in this file's device memory, which every GPU that loads
 * the library keeps until the process exits.
 *
 * The array's address is resolved once per device, on the first call made
 * on that device with the device current; that first call should therefore
 * come before any CUDA stream capture.  The resolved address is kept for
 * the life of the process: a cudaDeviceReset() of a device after its first
 * call is not supported (the next context would need the address resolved
 * again).  Every call shares the array and clears the rows it uses before
 * its own kernels run, so calls whose work overlaps on the GPU (other
 * streams, or other host threads on the same device) race on it and must be
 * serialised by the caller.
 *
 * Alignment: every pointer must be aligned to its element (4 bytes).  The
 * classifier rows are read as float4 only when dim % 4 == 0 and `weights`
 * is 16-byte aligned; any other 4-byte-aligned arena pointer takes the
 * scalar loop, so no caller alignment beyond the element is required.
 */
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include <cuda_runtime.h>

#include "../../include/nutllm_cuda.h"
#include "common.cuh"
#include "kernels.h"

namespace {

/* Largest batch one call may use: one accumulator per batch row. */
constexpr int kMaxRows = NUT_GREEDY_HEAD_MAX_BATCH;

static __device__ __align__(256) unsigned long long g_head_keys[kMaxRows];

nut_status fail(nut_status s, const std::string &m) {
    nut::set_last_error(m);
    return s;
}

/* Device address of g_head_keys on each device (resolved once). */
std::mutex g_lock;
unsigned long long *g_keys_addr[64] = {};

nut_status keys_address(int device, unsigned long long **out) {
    if (device < 0 || device >= 64)
        return fail(NUT_RUNTIME_ERROR, "greedy head: device index out of range");
    std::lock_guard<std::mutex> guard(g_lock);
    if (g_keys_addr[device] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_head_keys);
        if (e != cudaSuccess)
            return fail(NUT_RUNTIME_ERROR,
                        std::string("cuda: scratch address: ") + cudaGetErrorString(e));
        g_keys_addr[device] = static_cast<unsigned long long *>(p);
    }
    *out = g_keys_addr[device];
    return NUT_OK;
}

__global__ void clear_keys(unsigned long long *keys, int rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows)
        keys[i] = 0ull;
}

/* One batch row per blockIdx.y: x = rmsnorm(hidden row, norm) in shared
 * memory, then one warp per classifier row (fp32 dot product), first-index
 * argmax folded into keys[row] with atomicMax. */
__global__ void __launch_bounds__(256)
head_kernel(const float *__restrict__ hidden, const float *__restrict__ norm,
            const float *__restrict__ weights, int vocab, int dim, int vec,
            float *__restrict__ logits, unsigned long long *keys) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    __shared__ unsigned long long best_key[8];
    float *xs = reinterpret_cast<float *>(xs4);
    const float *h = hidden + size_t(blockIdx.y) * dim;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        ss = fmaf(h[i], h[i], ss);
    const float total = nut::block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(dim) + nut::kEps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        xs[i] = h[i] * scale * norm[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    float *out = logits != nullptr ? logits + size_t(blockIdx.y) * vocab : nullptr;
    unsigned long long mine = 0ull;
    for (int r = blockIdx.x * warps + warp; r < vocab; r += gridDim.x * warps) {
        const float *row = weights + size_t(r) * dim;
        float acc = 0.0f;
        if (vec) {
            const float4 *row4 = reinterpret_cast<const float4 *>(row);
            for (int g = lane; g < dim / 4; g += 32) {
                const float4 w = __ldg(row4 + g);
                const float4 x = xs4[g];
                acc = fmaf(w.x, x.x, acc);
                acc = fmaf(w.y, x.y, acc);
                acc = fmaf(w.z, x.z, acc);
                acc = fmaf(w.w, x.w, acc);
            }
        } else {
            for (int c = lane; c < dim; c += 32)
                acc = fmaf(row[c], xs[c], acc);
        }
        acc = nut::warp_sum(acc);
        if (lane == 0) {
            if (out != nullptr)
                out[r] = acc;
            const unsigned long long k = nut::argmax_key(acc, uint32_t(r));
            mine = k > mine ? k : mine;
        }
    }
    if (lane == 0)
        best_key[warp] = mine;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < warps; w++)
            b = best_key[w] > b ? best_key[w] : b;
        if (b != 0ull)
            atomicMax(keys + blockIdx.y, b);
    }
}

__global__ void keys_to_index(const unsigned long long *keys, int rows, int32_t *argmax) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows)
        argmax[i] = int32_t(nut::argmax_index(keys[i]));
}

} // namespace

extern "C" nut_status nut_greedy_head_static(const float *hidden, const float *final_norm,
                                             const float *weights, int64_t batch,
                                             int64_t vocab, int64_t dim, float *logits,
                                             int32_t *argmax, void *stream) {
    if (hidden == nullptr || final_norm == nullptr || weights == nullptr || argmax == nullptr)
        return fail(NUT_INVALID_ARGUMENT, "greedy head: null pointer");
    if (batch <= 0 || vocab <= 0 || dim <= 0)
        return fail(NUT_INVALID_ARGUMENT, "greedy head: invalid dimensions");
    if (batch > kMaxRows)
        return fail(NUT_LENGTH_ERROR,
                    "greedy head: batch " + std::to_string(batch) +
                        " exceeds the static scratch limit of " + std::to_string(kMaxRows));
    if (vocab > (int64_t(1) << 30) || dim > (1 << 14))
        return fail(NUT_LENGTH_ERROR, "greedy head: dimensions exceed device limits");
    auto misaligned = [](const void *p, uintptr_t a) {
        return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0;
    };
    if (misaligned(hidden, 4) || misaligned(final_norm, 4) || misaligned(weights, 4) ||
        misaligned(logits, 4) || misaligned(argmax, 4))
        return fail(NUT_INVALID_ARGUMENT, "greedy head: pointer not aligned to its element");
    /* float4 rows need 16-byte row starts: dim % 4 == 0 and an aligned base */
    const int vec = (dim % 4 == 0 && !misaligned(weights, 16)) ? 1 : 0;
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess)
        return fail(NUT_RUNTIME_ERROR, std::string("cuda: get device: ") + cudaGetErrorString(e));
    unsigned long long *keys = nullptr;
    const nut_status st = keys_address(device, &keys);
    if (st != NUT_OK)
        return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int rows = int(batch);
    clear_keys<<<(rows + 255) / 256, 256, 0, s>>>(keys, rows);
    const size_t smem = size_t((dim + 3) / 4) * 16;
    if (smem > 48 * 1024) {
        e = cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 int(smem));
        if (e != cudaSuccess)
            return fail(NUT_RUNTIME_ERROR, std::string("cuda: ") + cudaGetErrorString(e));
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const int per_row = int(std::min<int64_t>((vocab + 7) / 8, int64_t(4) * sms));
    head_kernel<<<dim3(per_row, rows), 256, smem, s>>>(hidden, final_norm, weights, int(vocab),
                                                        int(dim), vec, logits, keys);
    keys_to_index<<<(rows + 255) / 256, 256, 0, s>>>(keys, rows, argmax);
    nut::count_launches(3);
    e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(NUT_RUNTIME_ERROR, std::string("cuda: greedy head launch: ") +
                                           cudaGetErrorString(e));
    return NUT_OK;
}
