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
 *   attention_prefill causal GQA attention of every (token, head)
 *                     (attention_step, src/quant_model.cpp:68-105) in tiles
 *                     that share their keys and values, context rounded to
 *                     fp16 for the output projection
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

/* Causal attention of the prompt rows, tiled (attention_step,
 * src/quant_model.cpp:68-105, for every prompt token and head at once).
 *
 * CTA (tile, kv head g, sequence) owns kTileRows (token, head) rows: the
 * G = heads / kv_heads query heads of group g for QT = kTileRows / G
 * consecutive tokens, i.e. every row of the tile reads the same keys and
 * values.  Those are staged once per CTA, 32 PPL positions at a time, in a
 * double-buffered shared-memory ring (16-byte cp.async), and used by all 64
 * rows.  Warp w takes rows 8 w .. 8 w + 7:
 *   scores  lane j holds positions c0 + j and, with PPL = 2, c0 + j + 32
 *           for the warp's 8 rows (key rows padded to hd + 4 floats and read
 *           as float4: the 8 lanes of a quarter-warp hit distinct 16-byte
 *           bank groups when hd is a multiple of 8; query rows broadcast as
 *           float4);
 *   softmax online per row: chunk maximum by shuffles, the running
 *           maximum, exp weights (0 past the row's own position), the
 *           lane's share of the exp sum, the context rescaled;
 *   context lane owns dims lane, lane + 32, ... (DPL of them), weights
 *           broadcast from the warp's slice of shared memory.
 * After the last chunk the exp sums are reduced across lanes and the
 * context row is divided by it and rounded to fp16.  HD > 0 fixes the head
 * dim at compile time (the dot products unroll fully); HD = 0 takes it at
 * run time (up to 128).  fp32 throughout; the summation order differs from
 * the reference's double sums only by rounding.  Tiles with the longest
 * histories are scheduled first.  Measured (ncu, one launch at TinyLlama's
 * shape, 512 tokens): 86 us, ~1.9 warp instructions per warp FMA at 60 %
 * issue-active while SMs are busy, 34 % SM throughput over the launch (the
 * CTAs' work grows with their tokens' positions, so the last tiles finish
 * alone); shared memory and L2 are not the limit. */
constexpr int kTileRows = 64;
constexpr int kTileWarps = 8;
constexpr int kWarpRows = kTileRows / kTileWarps; /* 8 */

__device__ __forceinline__ void cp_async16(float *dst, const float *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <int HD, int PPL>
__global__ void __launch_bounds__(kTileWarps * 32)
attention_tiles_kernel(float *qkv, int ldq, int n, int seq0, int cache_seqs, int start,
                       const float *kcache, const float *vcache, int layer, int heads,
                       int kv_heads, int hd_rt, int max_seq, int Kp, __half *ctx, int zero_q) {
    constexpr int DPL = HD > 0 ? (HD + 31) / 32 : 4; /* context dims per lane */
    constexpr int CHUNK = 32 * PPL;                  /* positions per stage */
    extern __shared__ __align__(16) float att_smem[];
    const int hd = HD > 0 ? HD : hd_rt;
    const int G = heads / kv_heads, QT = kTileRows / G;
    const int ntiles = (n + QT - 1) / QT;
    const int tile = ntiles - 1 - int(blockIdx.x); /* longest histories first */
    const int g = int(blockIdx.y), sq = int(blockIdx.z);
    const int t0 = tile * QT, nt = min(QT, n - t0), R = nt * G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ldk = hd + 4, q4n = hd / 4;
    float *Qs = att_smem;                       /* [kTileRows][hd] */
    float *Ks = Qs + kTileRows * hd;            /* [2][CHUNK][hd + 4] */
    float *Vs = Ks + 2 * CHUNK * ldk;           /* [2][CHUNK][hd] */
    float *Ps = Vs + 2 * CHUNK * hd;            /* [kTileWarps][kWarpRows][CHUNK] */
    const size_t base =
        ((size_t(layer) * cache_seqs + size_t(seq0 + sq)) * kv_heads + g) * size_t(max_seq) * hd;
    /* positions 0 .. P - 1 cover every row of the tile */
    const int P = start + t0 + nt, nch = (P + CHUNK - 1) / CHUNK;
    auto stage = [&](int c) {
        const int buf = c & 1, j0 = c * CHUNK;
        float *kd = Ks + buf * CHUNK * ldk, *vd = Vs + buf * CHUNK * hd;
        /* rows past P repeat row P - 1 (finite values; their weights are 0) */
        for (int i = threadIdx.x; i < CHUNK * q4n; i += kTileWarps * 32) {
            const int jj = i / q4n, d = (i - jj * q4n) * 4;
            const size_t off = base + size_t(min(j0 + jj, P - 1)) * hd + d;
            cp_async16(kd + jj * ldk + d, kcache + off);
            cp_async16(vd + jj * hd + d, vcache + off);
        }
        cp_async_commit();
    };
    stage(0);
    /* the tile's query rows (row i: token t0 + i / G, head g G + i % G) */
    for (int i = threadIdx.x; i < kTileRows * q4n; i += kTileWarps * 32) {
        const int r = i / q4n, d = (i - r * q4n) * 4;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r < R) {
            const int t = t0 + r / G, h = g * G + r % G;
            float *src = qkv + (size_t(sq) * n + t) * ldq + h * hd + d;
            v = *reinterpret_cast<const float4 *>(src);
            if (zero_q) /* consumed: the next split-K GEMM adds into it */
                *reinterpret_cast<float4 *>(src) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        *reinterpret_cast<float4 *>(Qs + r * hd + d) = v;
    }
    const float scale = 1.0f / sqrtf(float(hd));
    const int r0 = warp * kWarpRows;
    /* the last position any row of this warp attends to (-1: no live row) */
    const int wmax = r0 < R ? start + t0 + min(R - 1, r0 + kWarpRows - 1) / G : -1;
    float m[kWarpRows], l[kWarpRows], acc[kWarpRows][DPL];
#pragma unroll
    for (int r = 0; r < kWarpRows; r++) {
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int k = 0; k < DPL; k++)
            acc[r][k] = 0.0f;
    }
    float *pw = Ps + warp * kWarpRows * CHUNK;
    for (int c = 0; c < nch; c++) {
        if (c + 1 < nch) {
            stage(c + 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int buf = c & 1, c0 = c * CHUNK;
        if (c0 <= wmax) {
            float s[PPL][kWarpRows];
#pragma unroll
            for (int u = 0; u < PPL; u++)
#pragma unroll
                for (int r = 0; r < kWarpRows; r++)
                    s[u][r] = 0.0f;
            const float *kb = Ks + buf * CHUNK * ldk + lane * ldk;
#pragma unroll(HD > 0 ? HD / 4 : 4)
            for (int d = 0; d < hd; d += 4) {
                float4 k4[PPL];
#pragma unroll
                for (int u = 0; u < PPL; u++)
                    k4[u] = *reinterpret_cast<const float4 *>(kb + u * 32 * ldk + d);
#pragma unroll
                for (int r = 0; r < kWarpRows; r++) {
                    const float4 q = *reinterpret_cast<const float4 *>(Qs + (r0 + r) * hd + d);
#pragma unroll
                    for (int u = 0; u < PPL; u++) {
                        s[u][r] = fmaf(q.x, k4[u].x, s[u][r]);
                        s[u][r] = fmaf(q.y, k4[u].y, s[u][r]);
                        s[u][r] = fmaf(q.z, k4[u].z, s[u][r]);
                        s[u][r] = fmaf(q.w, k4[u].w, s[u][r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < kWarpRows; r++) {
                const int row = r0 + r;
                const int last = row < R ? start + t0 + row / G : -1;
                float sc[PPL], mx = -INFINITY;
#pragma unroll
                for (int u = 0; u < PPL; u++) {
                    sc[u] = c0 + u * 32 + lane <= last ? s[u][r] * scale : -INFINITY;
                    mx = fmaxf(mx, sc[u]);
                }
                const float mn = fmaxf(m[r], warp_max(mx));
                float corr = 1.0f, lsum = 0.0f;
                if (mn != -INFINITY) {
                    corr = expf(m[r] - mn); /* 0 while m is still -inf */
#pragma unroll
                    for (int u = 0; u < PPL; u++) {
                        sc[u] = expf(sc[u] - mn); /* 0 past the row's position */
                        lsum += sc[u];
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < PPL; u++)
                        sc[u] = 0.0f;
                }
                l[r] = fmaf(l[r], corr, lsum);
#pragma unroll
                for (int k = 0; k < DPL; k++)
                    acc[r][k] *= corr;
                m[r] = mn;
#pragma unroll
                for (int u = 0; u < PPL; u++)
                    pw[r * CHUNK + u * 32 + lane] = sc[u];
            }
            __syncwarp();
            const float *vb = Vs + buf * CHUNK * hd;
#pragma unroll 2
            for (int jj = 0; jj < CHUNK; jj += 4) {
                float v[4][DPL];
#pragma unroll
                for (int u = 0; u < 4; u++)
#pragma unroll
                    for (int k = 0; k < DPL; k++) {
                        const int d = lane + 32 * k;
                        v[u][k] = d < hd ? vb[(jj + u) * hd + d] : 0.0f;
                    }
#pragma unroll
                for (int r = 0; r < kWarpRows; r++) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(pw + r * CHUNK + jj);
#pragma unroll
                    for (int k = 0; k < DPL; k++) {
                        acc[r][k] = fmaf(p4.x, v[0][k], acc[r][k]);
                        acc[r][k] = fmaf(p4.y, v[1][k], acc[r][k]);
                        acc[r][k] = fmaf(p4.z, v[2][k], acc[r][k]);
                        acc[r][k] = fmaf(p4.w, v[3][k], acc[r][k]);
                    }
                }
            }
            __syncwarp(); /* the weights are rewritten by the next chunk */
        }
        __syncthreads(); /* buffer c & 1 is restaged by chunk c + 2 */
    }
#pragma unroll
    for (int r = 0; r < kWarpRows; r++) {
        const int row = r0 + r;
        const float total = warp_sum(l[r]);
        if (row >= R)
            continue;
        const int t = t0 + row / G, h = g * G + row % G;
        __half *out = ctx + (size_t(sq) * n + t) * Kp + h * hd;
        const float inv = 1.0f / total;
#pragma unroll
        for (int k = 0; k < DPL; k++) {
            const int d = lane + 32 * k;
            if (d < hd)
                out[d] = to_half_sat(acc[r][k] * inv);
        }
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

bool attention_prefill_supported(int heads, int kv_heads, int hd, int ldq) {
    if (kv_heads <= 0 || heads % kv_heads != 0)
        return false;
    const int G = heads / kv_heads;
    return G <= kTileRows && kTileRows % G == 0 && hd > 0 && hd % 4 == 0 && hd <= 128 &&
           ldq % 4 == 0;
}

template <int HD, int PPL>
cudaError_t launch_tiles(float *qkv, int n, int nseq, int ldq, int seq0, int cache_seqs,
                         int start, const float *kcache, const float *vcache, int layer,
                         int heads, int kv_heads, int hd, int max_seq, int Kp, __half *ctx,
                         int zero_q, cudaStream_t s) {
    constexpr int CHUNK = 32 * PPL;
    const size_t smem = (size_t(kTileRows) * hd + size_t(2 * CHUNK) * (hd + 4) +
                         size_t(2 * CHUNK) * hd + size_t(kTileRows) * CHUNK) *
                        sizeof(float);
    auto k = attention_tiles_kernel<HD, PPL>;
    const cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess)
        return e;
    const int QT = kTileRows / (heads / kv_heads);
    const dim3 grid((n + QT - 1) / QT, kv_heads, nseq);
    k<<<grid, kTileWarps * 32, smem, s>>>(qkv, ldq, n, seq0, cache_seqs, start, kcache, vcache,
                                          layer, heads, kv_heads, hd, max_seq, Kp, ctx, zero_q);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t attention_prefill(float *qkv, int n, int nseq, int ldq, int seq0, int cache_seqs,
                              int start, const float *kcache, const float *vcache, int layer,
                              int heads, int kv_heads, int hd, int max_seq, int Kp,
                              uint16_t *ctx, bool zero_q, cudaStream_t s) {
    if (!attention_prefill_supported(heads, kv_heads, hd, ldq) || n <= 0 || nseq <= 0 ||
        nseq > 65535 || start < 0 || start + n > max_seq)
        return cudaErrorInvalidValue;
    auto *c = reinterpret_cast<__half *>(ctx);
    const int zq = zero_q ? 1 : 0;
    /* compile-time head dims of the common shapes; two positions per lane
     * where the staging ring of 64 positions leaves room for two CTAs per
     * SM (hd <= 64) */
    switch (hd) {
    case 32:
        return launch_tiles<32, 2>(qkv, n, nseq, ldq, seq0, cache_seqs, start, kcache, vcache,
                                   layer, heads, kv_heads, hd, max_seq, Kp, c, zq, s);
    case 48:
        return launch_tiles<48, 2>(qkv, n, nseq, ldq, seq0, cache_seqs, start, kcache, vcache,
                                   layer, heads, kv_heads, hd, max_seq, Kp, c, zq, s);
    case 64:
        return launch_tiles<64, 2>(qkv, n, nseq, ldq, seq0, cache_seqs, start, kcache, vcache,
                                   layer, heads, kv_heads, hd, max_seq, Kp, c, zq, s);
    case 128:
        return launch_tiles<128, 1>(qkv, n, nseq, ldq, seq0, cache_seqs, start, kcache, vcache,
                                    layer, heads, kv_heads, hd, max_seq, Kp, c, zq, s);
    default:
        return launch_tiles<0, 1>(qkv, n, nseq, ldq, seq0, cache_seqs, start, kcache, vcache,
                                  layer, heads, kv_heads, hd, max_seq, Kp, c, zq, s);
    }
}

cudaError_t zero_tail(uint16_t *x, int M, int dim, int Kp, cudaStream_t s) {
    if (Kp <= dim)
        return cudaSuccess;
    zero_tail_kernel<<<blocks_for(int64_t(M) * (Kp - dim), 256), 256, 0, s>>>(
        reinterpret_cast<__half *>(x), M, dim, Kp);
    count_launches(1);
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
