/* Batched prefill: the prompt's tokens through every layer at once.
 *
 * prefill_quantized (src/quant_model.cpp:208-220) runs decode_quantized_token
 * for each prompt token in turn.  Every projection then multiplies the same
 * weights by one vector per token, so the whole prompt is one dense
 * contraction per projection: this file holds the row-wise operations
 * between those GEMMs (gemm_tc.cu), for M prompt tokens at positions
 * start .. start + M - 1:
 *   gather_rows       h[m] = embedding row of token m
 *   rmsnorm_rows      x[m] = fp16(rmsnorm(h[m]) * weight) (src/ops.cpp:111-134)
 *   rope_kv_rows      RoPE on the q and k rows in place (the reference's
 *                     unfused products, src/quant_model.cpp:26-37) and the
 *                     k, v rows appended to the KV cache
 *   attention_rows    causal GQA attention of every (token, head)
 *                     (attention_step, src/quant_model.cpp:68-105), context
 *                     rounded to fp16 for the output projection
 *   swiglu_rows       a = fp16(silu(gate) * up) (src/ops.cpp:136-138) from the
 *                     gate/up GEMM's rows interleaved in groups of 8
 * fp16 conversions round to nearest and saturate at +-65504.
 */
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "prefill.h"

namespace nut {
namespace {

__device__ __forceinline__ __half to_half_sat(float v) {
    return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}

__global__ void gather_rows_kernel(const float *emb, const int32_t *tokens, int M, int dim,
                                   int vocab, float *h) {
    const int m = blockIdx.x;
    if (m >= M)
        return;
    const int t = tokens[m];
    const bool ok = t >= 0 && t < vocab;
    for (int k = threadIdx.x; k < dim; k += blockDim.x)
        h[size_t(m) * dim + k] = ok ? emb[size_t(t) * dim + k] : 0.0f;
}

__global__ void rmsnorm_rows_kernel(const float *h, const float *w, int dim, int Kp,
                                    __half *out) {
    __shared__ float red[32];
    const int m = blockIdx.x;
    const float *x = h + size_t(m) * dim;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < dim; k += blockDim.x)
        ss = fmaf(x[k], x[k], ss);
    const float total = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(dim) + kEps);
    __half *o = out + size_t(m) * Kp;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x)
        o[k] = to_half_sat(k < dim ? x[k] * scale * w[k] : 0.0f);
}

/* One thread per (row m, rotation pair or value element). */
__global__ void rope_kv_rows_kernel(float *qkv, int M, int ldq, int start, const float *rope_cos,
                                    const float *rope_sin, int heads, int kv_heads, int hd,
                                    int dim, int kvd, float *kcache, float *vcache, int layer,
                                    int max_seq) {
    const int half = hd / 2;
    const int per_row = heads * half + kv_heads * half + kvd;
    const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= int64_t(M) * per_row)
        return;
    const int m = int(gid / per_row), r = int(gid - int64_t(m) * per_row);
    const int pos = start + m;
    float *row = qkv + size_t(m) * ldq;
    const float *cs = rope_cos + size_t(pos) * half, *sn = rope_sin + size_t(pos) * half;
    if (r < heads * half) {                       /* query pair */
        const int h = r / half, i = r - h * half;
        float *p = row + h * hd + 2 * i;
        const float a = p[0], b = p[1];
        p[0] = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(b, sn[i]));
        p[1] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(b, cs[i]));
        return;
    }
    const int r2 = r - heads * half;
    if (r2 < kv_heads * half) {                   /* key pair: rotate, append */
        const int h = r2 / half, i = r2 - h * half;
        float *p = row + dim + h * hd + 2 * i;
        const float a = p[0], b = p[1];
        const float x0 = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(b, sn[i]));
        const float x1 = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(b, cs[i]));
        p[0] = x0;
        p[1] = x1;
        float *kc = kcache + ((size_t(layer) * kv_heads + h) * max_seq + pos) * hd + 2 * i;
        kc[0] = x0;
        kc[1] = x1;
        return;
    }
    const int e = r2 - kv_heads * half;           /* value element */
    const int h = e / hd, d = e - h * hd;
    vcache[((size_t(layer) * kv_heads + h) * max_seq + pos) * hd + d] = row[dim + kvd + e];
}

/* One warp per (token m, head h); 4 warps per CTA.  Positions 0 .. start+m:
 * scores (a lane per position) into the warp's shared buffer, max and
 * exp-sum by shuffles, then the context with each lane owning dims lane,
 * lane + 32, ... */
constexpr int kAttWarps = 4;

__global__ void __launch_bounds__(kAttWarps * 32)
attention_rows_kernel(const float *qkv, int M, int ldq, int start, const float *kcache,
                      const float *vcache, int layer, int heads, int kv_heads, int hd, int dim,
                      int max_seq, int Kp, __half *ctx) {
    extern __shared__ float att_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t item = int64_t(blockIdx.x) * kAttWarps + warp;
    if (item >= int64_t(M) * heads)
        return;
    const int m = int(item / heads), h = int(item - int64_t(m) * heads);
    const int npos = start + m + 1;
    float *q = att_smem + size_t(warp) * (hd + max_seq);
    float *w = q + hd;
    const float *qsrc = qkv + size_t(m) * ldq + h * hd;
    for (int d = lane; d < hd; d += 32)
        q[d] = qsrc[d];
    __syncwarp();
    const int g = h / (heads / kv_heads);
    const size_t base = (size_t(layer) * kv_heads + g) * size_t(max_seq) * hd;
    const float scale = 1.0f / sqrtf(float(hd));
    float mx = -INFINITY;
    for (int j = lane; j < npos; j += 32) {
        const float *kj = kcache + base + size_t(j) * hd;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        int d = 0;
        for (; d + 4 <= hd; d += 4) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kj + d);
            a0 = fmaf(q[d], k4.x, a0);
            a1 = fmaf(q[d + 1], k4.y, a1);
            a2 = fmaf(q[d + 2], k4.z, a2);
            a3 = fmaf(q[d + 3], k4.w, a3);
        }
        for (; d < hd; d++)
            a0 = fmaf(q[d], kj[d], a0);
        const float sc = ((a0 + a1) + (a2 + a3)) * scale;
        w[j] = sc;
        mx = fmaxf(mx, sc);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
    for (int j = lane; j < npos; j += 32) {
        const float e = expf(w[j] - mx);
        w[j] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    const float inv = 1.0f / sum;
    __half *out = ctx + size_t(m) * Kp + h * hd;
    for (int d = lane; d < hd; d += 32) {
        const float *vd = vcache + base + d;
        float c = 0.0f;
        for (int j = 0; j < npos; j++)
            c = fmaf(w[j], vd[size_t(j) * hd], c);
        out[d] = to_half_sat(c * inv);
    }
}

__global__ void zero_tail_kernel(__half *x, int M, int dim, int Kp) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int tail = Kp - dim;
    if (tail <= 0 || i >= int64_t(M) * tail)
        return;
    const int64_t m = i / tail;
    x[m * Kp + dim + (i - m * tail)] = to_half_sat(0.0f);
}

__global__ void swiglu_rows_kernel(const float *gu, int M, int ffn, int Kp, __half *act,
                                   int clear) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= int64_t(M) * Kp)
        return;
    const int64_t m = i / Kp;
    const int u = int(i - m * Kp);
    float a = 0.0f;
    if (u < ffn) {
        float *row = const_cast<float *>(gu) + size_t(m) * 2 * ffn;
        const float gte = row[(u / 8) * 16 + (u % 8)];
        const float up = row[(u / 8) * 16 + 8 + (u % 8)];
        a = gte / (1.0f + expf(-gte)) * up;
        if (clear) { /* each gate/up value has one reader: zero it for the
                        next GEMM that adds into the rows */
            row[(u / 8) * 16 + (u % 8)] = 0.0f;
            row[(u / 8) * 16 + 8 + (u % 8)] = 0.0f;
        }
    }
    act[i] = to_half_sat(a);
}

inline int blocks_for(int64_t n, int t) { return int((n + t - 1) / t); }

} // namespace

cudaError_t gather_rows(const float *emb, const int32_t *tokens, int M, int dim, int vocab,
                        float *h, cudaStream_t s) {
    gather_rows_kernel<<<M, 256, 0, s>>>(emb, tokens, M, dim, vocab, h);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t rmsnorm_rows(const float *h, const float *w, int M, int dim, int Kp, uint16_t *out,
                         cudaStream_t s) {
    rmsnorm_rows_kernel<<<M, 256, 0, s>>>(h, w, dim, Kp,
                                          reinterpret_cast<__half *>(out));
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t rope_kv_rows(float *qkv, int M, int ldq, int start, const float *rope_cos,
                         const float *rope_sin, int heads, int kv_heads, int hd, int dim, int kvd,
                         float *kcache, float *vcache, int layer, int max_seq, cudaStream_t s) {
    const int64_t n = int64_t(M) * (heads * (hd / 2) + kv_heads * (hd / 2) + kvd);
    rope_kv_rows_kernel<<<blocks_for(n, 256), 256, 0, s>>>(qkv, M, ldq, start, rope_cos,
                                                           rope_sin, heads, kv_heads, hd, dim,
                                                           kvd, kcache, vcache, layer, max_seq);
    count_launches(1);
    return cudaGetLastError();
}

size_t attention_rows_smem(int hd, int max_seq) {
    return size_t(kAttWarps) * size_t(hd + max_seq) * sizeof(float);
}

cudaError_t attention_rows(const float *qkv, int M, int ldq, int start, const float *kcache,
                           const float *vcache, int layer, int heads, int kv_heads, int hd,
                           int dim, int max_seq, int Kp, uint16_t *ctx, cudaStream_t s) {
    const size_t smem = attention_rows_smem(hd, max_seq);
    cudaError_t e = cudaFuncSetAttribute(attention_rows_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess)
        return e;
    auto *c = reinterpret_cast<__half *>(ctx);
    const int64_t items = int64_t(M) * heads;
    attention_rows_kernel<<<blocks_for(items, kAttWarps), kAttWarps * 32, smem, s>>>(
        qkv, M, ldq, start, kcache, vcache, layer, heads, kv_heads, hd, dim, max_seq, Kp, c);
    zero_tail_kernel<<<blocks_for(int64_t(M) * (Kp > dim ? Kp - dim : 1), 256), 256, 0, s>>>(
        c, M, dim, Kp);
    count_launches(2);
    return cudaGetLastError();
}

cudaError_t swiglu_rows(const float *gu, int M, int ffn, int Kp, uint16_t *act, cudaStream_t s,
                        bool clear_src) {
    swiglu_rows_kernel<<<blocks_for(int64_t(M) * Kp, 256), 256, 0, s>>>(
        gu, M, ffn, Kp, reinterpret_cast<__half *>(act), clear_src ? 1 : 0);
    count_launches(1);
    return cudaGetLastError();
}

} // namespace nut
