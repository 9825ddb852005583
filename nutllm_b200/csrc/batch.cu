/* Row kernels of the batched decode step (batch.h).
 *
 * The batch advances B independent sequences by one token per step through
 * the same quantised decoder as decode_quantized_token
 * (src/quant_model.cpp:158-206); the projections are GEMMs over the B rows
 * (gemm_tc.cu) and these kernels do the work between them. */
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "batch.h"
#include "common.cuh"
#include "kernels.h"

namespace nut {
namespace {

__device__ __forceinline__ __half to_half_sat(float v) {
    return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}

inline int blocks_for(int64_t n, int t) { return int((n + t - 1) / t); }

__global__ void add_rmsnorm_rows_kernel(float *h, const float *part, const float *w, int dim,
                                        int Kp, __half *out) {
    __shared__ float red[32];
    const int b = blockIdx.x;
    float *x = h + size_t(b) * dim;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        float v = x[k];
        if (part != nullptr) {
            v += part[size_t(b) * dim + k];
            x[k] = v;
        }
        ss = fmaf(v, v, ss);
    }
    const float total = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(dim) + kEps);
    __half *o = out + size_t(b) * Kp;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x)
        o[k] = to_half_sat(k < dim ? x[k] * scale * w[k] : 0.0f);
}

/* One thread per (sequence b, rotation pair or value element). */
__global__ void rope_kv_batch_kernel(float *qkv, int B, int ldq, const int *pos_p,
                                     const float *rope_cos, const float *rope_sin, int heads,
                                     int kv_heads, int hd, float *kcache, float *vcache,
                                     int layer, int max_seq) {
    const int half = hd / 2, dq = heads * hd, kvd = kv_heads * hd;
    const int per_row = heads * half + kv_heads * half + kvd;
    const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= int64_t(B) * per_row)
        return;
    const int pos = *pos_p;
    const int b = int(gid / per_row), r = int(gid - int64_t(b) * per_row);
    float *row = qkv + size_t(b) * ldq;
    const float *cs = rope_cos + size_t(pos) * half, *sn = rope_sin + size_t(pos) * half;
    const size_t seq = (size_t(layer) * B + b) * kv_heads;
    if (r < heads * half) {                       /* query pair */
        const int h = r / half, i = r - h * half;
        float *p = row + h * hd + 2 * i;
        const float a = p[0], c = p[1];
        p[0] = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(c, sn[i]));
        p[1] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(c, cs[i]));
        return;
    }
    const int r2 = r - heads * half;
    if (r2 < kv_heads * half) {                   /* key pair: rotate, append */
        const int h = r2 / half, i = r2 - h * half;
        float *p = row + dq + h * hd + 2 * i;
        const float a = p[0], c = p[1];
        const float x0 = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(c, sn[i]));
        const float x1 = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(c, cs[i]));
        p[0] = x0;
        p[1] = x1;
        float *kc = kcache + ((seq + h) * max_seq + pos) * hd + 2 * i;
        kc[0] = x0;
        kc[1] = x1;
        return;
    }
    const int e = r2 - kv_heads * half;           /* value element */
    const int h = e / hd, d = e - h * hd;
    vcache[((seq + h) * max_seq + pos) * hd + d] = row[dq + kvd + e];
}

/* One CTA of kAttWarps warps per (sequence, head).  A cached row of hd
 * floats is read by `lpr` lanes (the largest power of two dividing hd / 4;
 * float4 each, hd / (4 lpr) chunks per lane), so a warp covers 32 / lpr
 * positions per iteration and every row read is coalesced.  Scores go to shared memory, the softmax is
 * CTA-wide, and the context is accumulated per warp over its positions
 * (float4 per lane) and summed across the warps. */
constexpr int kAttWarps = 4;

__global__ void __launch_bounds__(kAttWarps * 32)
attention_batch_kernel(const float *qkv, int B, int ldq, const int *pos_p, const float *kcache,
                       const float *vcache, int layer, int heads, int kv_heads, int hd,
                       int max_seq, int Kp, __half *ctx) {
    extern __shared__ float sm[];
    float *q = sm;                       /* [hd] */
    float *part = q + hd;                /* [kAttWarps][hd] */
    float *w = part + kAttWarps * hd;    /* [max_seq] */
    __shared__ float red[32];
    const int b = blockIdx.x / heads, h = blockIdx.x - b * heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npos = *pos_p + 1;
    const int g = h / (heads / kv_heads);
    const size_t base = ((size_t(layer) * B + b) * kv_heads + g) * size_t(max_seq) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x)
        q[d] = qkv[size_t(b) * ldq + h * hd + d];
    __syncthreads();
    const int chunks = hd / 4;                       /* float4 per row */
    int lpr = 32;                                    /* lanes per row: the largest */
    while (chunks % lpr != 0)                        /* power of two dividing chunks */
        lpr >>= 1;
    const int cpl = chunks / lpr;                    /* chunks per lane (<= 8) */
    const int rpi = 32 / lpr;                        /* rows per warp iteration */
    const int sub = lane / lpr, li = lane - sub * lpr;
    const float scale = 1.0f / sqrtf(float(hd));
    const float4 *q4 = reinterpret_cast<const float4 *>(q);
    float mx = -INFINITY;
    for (int j0 = warp * rpi; j0 < npos; j0 += kAttWarps * rpi) {
        const int j = j0 + sub;
        float a = 0.0f;
        if (j < npos) {
            const float4 *kj = reinterpret_cast<const float4 *>(kcache + base + size_t(j) * hd);
            for (int c = 0; c < cpl; c++) {
                const float4 k4 = kj[li + c * lpr], x4 = q4[li + c * lpr];
                a = fmaf(x4.x, k4.x, a);
                a = fmaf(x4.y, k4.y, a);
                a = fmaf(x4.z, k4.z, a);
                a = fmaf(x4.w, k4.w, a);
            }
        }
        for (int o = lpr >> 1; o > 0; o >>= 1)
            a += __shfl_xor_sync(0xffffffffu, a, o);
        if (li == 0 && j < npos) {
            const float sc = a * scale;
            w[j] = sc;
            mx = fmaxf(mx, sc);
        }
    }
    mx = block_max(mx, red);
    float sum = 0.0f;
    for (int j = threadIdx.x; j < npos; j += blockDim.x) {
        const float e = expf(w[j] - mx);
        w[j] = e;
        sum += e;
    }
    sum = block_sum(sum, red); /* its barriers also publish w[] */
    float4 acc[8];
#pragma unroll
    for (int c = 0; c < 8; c++)
        acc[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int j0 = warp * rpi; j0 < npos; j0 += kAttWarps * rpi) {
        const int j = j0 + sub;
        if (j < npos) {
            const float e = w[j];
            const float4 *vj = reinterpret_cast<const float4 *>(vcache + base + size_t(j) * hd);
#pragma unroll
            for (int c = 0; c < 8; c++)
                if (c < cpl) {
                    const float4 v4 = vj[li + c * lpr];
                    acc[c].x = fmaf(e, v4.x, acc[c].x);
                    acc[c].y = fmaf(e, v4.y, acc[c].y);
                    acc[c].z = fmaf(e, v4.z, acc[c].z);
                    acc[c].w = fmaf(e, v4.w, acc[c].w);
                }
        }
    }
    /* rows handled by different `sub` groups of the warp: fold them */
    for (int o = 16; o >= lpr; o >>= 1)
#pragma unroll
        for (int c = 0; c < 8; c++) {
            acc[c].x += __shfl_xor_sync(0xffffffffu, acc[c].x, o);
            acc[c].y += __shfl_xor_sync(0xffffffffu, acc[c].y, o);
            acc[c].z += __shfl_xor_sync(0xffffffffu, acc[c].z, o);
            acc[c].w += __shfl_xor_sync(0xffffffffu, acc[c].w, o);
        }
    if (sub == 0)
#pragma unroll
        for (int c = 0; c < 8; c++)
            if (c < cpl)
                reinterpret_cast<float4 *>(part + warp * hd)[li + c * lpr] = acc[c];
    __syncthreads();
    const float inv = 1.0f / sum;
    __half *out = ctx + size_t(b) * Kp + h * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float c = 0.0f;
        for (int k = 0; k < kAttWarps; k++)
            c += part[k * hd + d];
        out[d] = to_half_sat(c * inv);
    }
}

__global__ void zero_cols_kernel(__half *x, int B, int from, int Kp) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int tail = Kp - from;
    if (tail <= 0 || i >= int64_t(B) * tail)
        return;
    const int64_t b = i / tail;
    x[b * Kp + from + (i - b * tail)] = to_half_sat(0.0f);
}

__global__ void argmax_keys_kernel(const float *logits, int V, int v0, unsigned long long *keys) {
    __shared__ unsigned long long best[32];
    const int b = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float *row = logits + size_t(b) * V;
    unsigned long long k = 0ull;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const unsigned long long c = argmax_key(row[i], uint32_t(v0 + i));
        k = c > k ? c : k;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long c = __shfl_xor_sync(0xffffffffu, k, o);
        k = c > k ? c : k;
    }
    if (lane == 0)
        best[warp] = k;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0ull;
        for (int w = 0; w < int(blockDim.x >> 5); w++)
            m = best[w] > m ? best[w] : m;
        keys[b] = m;
    }
}

__global__ void keys_to_ids_kernel(const unsigned long long *keys, int B, int32_t *ids,
                                   int32_t *out, int ld, const int *step) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B)
        return;
    const int32_t t = int32_t(argmax_index(keys[b]));
    ids[b] = t;
    if (out != nullptr)
        out[size_t(b) * ld + *step] = t;
}

__global__ void prompt_column_kernel(const int32_t *prompts, int B, int n, const int *step,
                                     int32_t *ids) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B)
        ids[b] = prompts[size_t(b) * n + *step];
}

__global__ void advance_kernel(int *pos, int *step) {
    *pos += 1;
    *step += 1;
}

/* splitmix64 finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom
 * number generators", OOPSLA 2014): a counter-based hash, so every element
 * is generated independently of the others. */
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t element_hash(uint64_t seed, uint64_t stream, uint64_t i) {
    return mix64(seed ^ mix64(stream * 0xD1B54A32D192ED03ull + i));
}

__global__ void synth_normal_kernel(uint64_t seed, uint64_t stream, float sigma, float *out,
                                    size_t n) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    const uint64_t r = element_hash(seed, stream, i);
    /* Box-Muller from two 24-bit uniforms in (0, 1] and [0, 1) */
    const float u1 = (float(uint32_t(r >> 40)) + 1.0f) * (1.0f / 16777216.0f);
    const float u2 = float(uint32_t(r >> 8) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    out[i] = sigma * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void synth_int4_f16_kernel(uint64_t seed, uint64_t stream, float sigma, int rows,
                                      int cols, int ld, __half *out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(rows) * ld)
        return;
    const int r = int(i / ld), c = int(i - int64_t(r) * ld);
    if (c >= cols) {
        out[i] = __float2half_rn(0.0f);
        return;
    }
    const uint64_t hq = element_hash(seed, stream, uint64_t(r) * cols + c);
    const uint64_t hs = element_hash(seed, stream ^ 0x5CA1Eull, uint64_t(r) * cols + c / 32);
    const int q = int(hq % 15u) - 7;
    const float unit = sigma * 2.5f / 7.0f;
    const float s = __half2float(__float2half_rn(
        unit * (0.75f + 0.5f * float(uint32_t(hs >> 40)) * (1.0f / 16777216.0f))));
    out[i] = __float2half_rn(float(q) * s);
}

} // namespace

cudaError_t add_rmsnorm_rows(float *h, const float *part, const float *w, int B, int dim,
                             int Kp, uint16_t *out, cudaStream_t s) {
    add_rmsnorm_rows_kernel<<<B, 256, 0, s>>>(h, part, w, dim, Kp,
                                              reinterpret_cast<__half *>(out));
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t rope_kv_batch(float *qkv, int B, int ldq, const int *pos, const float *rope_cos,
                          const float *rope_sin, int heads, int kv_heads, int hd,
                          float *kcache, float *vcache, int layer, int max_seq,
                          cudaStream_t s) {
    const int64_t n = int64_t(B) * (heads * (hd / 2) + kv_heads * (hd / 2) + kv_heads * hd);
    rope_kv_batch_kernel<<<blocks_for(n, 256), 256, 0, s>>>(qkv, B, ldq, pos, rope_cos,
                                                            rope_sin, heads, kv_heads, hd,
                                                            kcache, vcache, layer, max_seq);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t attention_batch(const float *qkv, int B, int ldq, const int *pos,
                            const float *kcache, const float *vcache, int layer, int heads,
                            int kv_heads, int hd, int max_seq, int Kp, uint16_t *ctx,
                            cudaStream_t s) {
    /* float4 rows, at most 8 float4 per lane */
    if (hd % 4 != 0 || hd <= 0)
        return cudaErrorInvalidValue;
    int lpr = 32;
    while ((hd / 4) % lpr != 0)
        lpr >>= 1;
    if (hd / 4 / lpr > 8)
        return cudaErrorInvalidValue;
    const size_t smem = (size_t(hd) * (1 + kAttWarps) + size_t(max_seq)) * sizeof(float);
    if (smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            attention_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess)
            return e;
    }
    __half *c16 = reinterpret_cast<__half *>(ctx);
    attention_batch_kernel<<<B * heads, kAttWarps * 32, smem, s>>>(
        qkv, B, ldq, pos, kcache, vcache, layer, heads, kv_heads, hd, max_seq, Kp, c16);
    count_launches(1);
    if (Kp > heads * hd) {
        const int64_t n = int64_t(B) * (Kp - heads * hd);
        zero_cols_kernel<<<blocks_for(n, 256), 256, 0, s>>>(c16, B, heads * hd, Kp);
        count_launches(1);
    }
    return cudaGetLastError();
}

cudaError_t argmax_keys(const float *logits, int B, int V, int v0, unsigned long long *keys,
                        cudaStream_t s) {
    argmax_keys_kernel<<<B, 256, 0, s>>>(logits, V, v0, keys);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t keys_to_ids(const unsigned long long *keys, int B, int32_t *ids, int32_t *out,
                        int ld, const int *step, cudaStream_t s) {
    keys_to_ids_kernel<<<blocks_for(B, 128), 128, 0, s>>>(keys, B, ids, out, ld, step);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t prompt_column(const int32_t *prompts, int B, int n, const int *step, int32_t *ids,
                          cudaStream_t s) {
    prompt_column_kernel<<<blocks_for(B, 128), 128, 0, s>>>(prompts, B, n, step, ids);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t advance(int *pos, int *step, cudaStream_t s) {
    advance_kernel<<<1, 1, 0, s>>>(pos, step);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t synth_normal_dev(uint64_t seed, uint64_t stream, float sigma, float *out, size_t n,
                             cudaStream_t s) {
    synth_normal_kernel<<<blocks_for(int64_t(n), 256), 256, 0, s>>>(seed, stream, sigma, out, n);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t synth_int4_f16_dev(uint64_t seed, uint64_t stream, float sigma, int rows, int cols,
                               int ld, uint16_t *out, cudaStream_t s) {
    const int64_t n = int64_t(rows) * ld;
    synth_int4_f16_kernel<<<blocks_for(n, 256), 256, 0, s>>>(
        seed, stream, sigma, rows, cols, ld, reinterpret_cast<__half *>(out));
    count_launches(1);
    return cudaGetLastError();
}

} // namespace nut
