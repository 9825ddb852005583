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
#include "kernels_tc.h"

namespace nut {
namespace {

__device__ __forceinline__ __half to_half_sat(float v) {
    return __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f));
}

inline int blocks_for(int64_t n, int t) { return int((n + t - 1) / t); }

__global__ void add_rmsnorm_rows_kernel(float *h, float *part, int add, const float *w, int dim,
                                        int Kp, __half *out) {
    __shared__ float red[32];
    const int b = blockIdx.x;
    float *x = h + size_t(b) * dim;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < dim; k += blockDim.x) {
        float v = x[k];
        if (part != nullptr) {
            float *pk = part + size_t(b) * dim + k;
            if (add) {
                v += *pk;
                x[k] = v;
            }
            *pk = 0.0f; /* the next split-K GEMM adds into it */
        }
        ss = fmaf(v, v, ss);
    }
    const float total = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(dim) + kEps);
    __half *o = out + size_t(b) * Kp;
    for (int k = threadIdx.x; k < Kp; k += blockDim.x)
        o[k] = to_half_sat(k < dim ? x[k] * scale * w[k] : 0.0f);
}

/* The same row operation with the row held in registers: 256 threads,
 * float4 loads and stores, at most kNormVec float4 per thread (dim <=
 * 8192, dim % 4 == 0, 16-byte aligned rows, Kp % 2 == 0).  One read of h,
 * part and w, one write of h, part and out. */
constexpr int kNormThreads = 256;
constexpr int kNormVec = 8;

__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_rows_vec_kernel(float *h, float *part, int add, const float *w, int dim, int Kp,
                            __half *out) {
    __shared__ float red[32];
    const int b = blockIdx.x, n4 = dim / 4;
    float4 *x4 = reinterpret_cast<float4 *>(h + size_t(b) * dim);
    float4 *p4 = part != nullptr ? reinterpret_cast<float4 *>(part + size_t(b) * dim) : nullptr;
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    float4 v[kNormVec], g[kNormVec];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kNormVec; j++) {
        const int i = int(threadIdx.x) + j * kNormThreads;
        if (i < n4) {
            v[j] = x4[i];
            g[j] = w4[i];
            if (p4 != nullptr && add) {
                const float4 q = p4[i];
                v[j].x += q.x, v[j].y += q.y, v[j].z += q.z, v[j].w += q.w;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kNormVec; j++) {
        const int i = int(threadIdx.x) + j * kNormThreads;
        if (i < n4) {
            if (p4 != nullptr) {
                if (add)
                    x4[i] = v[j];
                p4[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f); /* the next split-K GEMM adds into it */
            }
            ss = fmaf(v[j].x, v[j].x, ss);
            ss = fmaf(v[j].y, v[j].y, ss);
            ss = fmaf(v[j].z, v[j].z, ss);
            ss = fmaf(v[j].w, v[j].w, ss);
        }
    }
    const float total = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(dim) + kEps);
    __half2 *o2 = reinterpret_cast<__half2 *>(out + size_t(b) * Kp);
#pragma unroll
    for (int j = 0; j < kNormVec; j++) {
        const int i = int(threadIdx.x) + j * kNormThreads;
        if (i < n4) {
            o2[2 * i] = __halves2half2(to_half_sat(v[j].x * scale * g[j].x),
                                       to_half_sat(v[j].y * scale * g[j].y));
            o2[2 * i + 1] = __halves2half2(to_half_sat(v[j].z * scale * g[j].z),
                                           to_half_sat(v[j].w * scale * g[j].w));
        }
    }
    const __half2 zero = __halves2half2(__float2half(0.0f), __float2half(0.0f));
    for (int k = dim / 2 + int(threadIdx.x); k < Kp / 2; k += kNormThreads)
        o2[k] = zero;
}

/* One thread per (sequence b, rotation pair or value element). */
__global__ void rope_kv_batch_kernel(float *qkv, int rows, int B, int ldq, const int *pos_p,
                                     const float *rope_cos, const float *rope_sin, int heads,
                                     int kv_heads, int hd, float *kcache, float *vcache,
                                     int layer, int max_seq, int pf_n, int seq0) {
    const int half = hd / 2, dq = heads * hd, kvd = kv_heads * hd;
    const int per_row = heads * half + kv_heads * half + kvd;
    const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= int64_t(rows) * per_row)
        return;
    const int b = int(gid / per_row), r = int(gid - int64_t(b) * per_row);
    /* decode: row b is sequence b at *pos; prefill: row b is position
     * b % pf_n of sequence seq0 + b / pf_n */
    const int pos = pf_n > 0 ? b % pf_n : *pos_p;
    const int sq = pf_n > 0 ? seq0 + b / pf_n : b;
    float *row = qkv + size_t(b) * ldq;
    const float *cs = rope_cos + size_t(pos) * half, *sn = rope_sin + size_t(pos) * half;
    const size_t seq = (size_t(layer) * B + sq) * kv_heads;
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
        p[0] = 0.0f; /* consumed: the next split-K GEMM adds into it */
        p[1] = 0.0f;
        float *kc = kcache + ((seq + h) * max_seq + pos) * hd + 2 * i;
        kc[0] = x0;
        kc[1] = x1;
        return;
    }
    const int e = r2 - kv_heads * half;           /* value element */
    const int h = e / hd, d = e - h * hd;
    vcache[((seq + h) * max_seq + pos) * hd + d] = row[dq + kvd + e];
    row[dq + kvd + e] = 0.0f;
}

/* One CTA of kAttWarps warps per (sequence, head), one pass over the
 * positions with a running (maximum, sum, context) per row group: a cached
 * row of hd floats is read by `lpr` lanes (the largest power of two
 * dividing hd / 4; float4 each, hd / (4 lpr) chunks per lane), so a warp
 * covers 32 / lpr positions per step and every row read is coalesced; U
 * steps' key rows, then their value rows, are in flight together.  The row
 * groups' states are merged at the end (m = max m_k, l = sum l_k e^(m_k -
 * m), context = sum c_k e^(m_k - m) / l), which equals the reference's
 * softmax over all positions up to rounding. */
constexpr int kAttWarps = 8;

template <int CPL>
__global__ void __launch_bounds__(kAttWarps * 32)
attention_batch_kernel(const float *qkv, int B, int ldq, const int *pos_p, const float *kcache,
                       const float *vcache, int layer, int heads, int kv_heads, int hd,
                       int max_seq, int Kp, __half *ctx) {
    extern __shared__ float sm[];
    /* row b is sequence b at *pos */
    const int b = blockIdx.x / heads, h = blockIdx.x - b * heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npos = *pos_p + 1;
    const int g = h / (heads / kv_heads);
    const size_t base = ((size_t(layer) * B + b) * kv_heads + g) * size_t(max_seq) * hd;
    const int lpr = hd / 4 / CPL;                    /* lanes per row (a power of two) */
    const int rpi = 32 / lpr;                        /* rows per warp step */
    const int sub = lane / lpr, li = lane - sub * lpr;
    const int nst = kAttWarps * rpi;                 /* row-group states */
    float *q = sm;                                   /* [hd] */
    float *st_c = q + hd;                            /* [nst][hd] */
    float *st_m = st_c + size_t(nst) * hd;           /* [nst] */
    float *st_l = st_m + nst;                        /* [nst] */
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float *src = const_cast<float *>(qkv) + size_t(b) * ldq + h * hd + d;
        q[d] = *src;
        *src = 0.0f; /* consumed: the next split-K GEMM adds into it */
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(float(hd));
    float4 qv[CPL], acc[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        qv[c] = reinterpret_cast<const float4 *>(q)[li + c * lpr];
        acc[c] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float m = -INFINITY, l = 0.0f;
    constexpr int U = 4;
    const int stride = kAttWarps * rpi;
    for (int j0 = warp * rpi; j0 < npos; j0 += U * stride) {
        /* the step's key and value rows, all loads issued together (rows
         * past the end read row 0 and are masked) */
        float4 kk[U][CPL], vv[U][CPL];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = j0 + u * stride + sub;
            const size_t off = base + size_t(j < npos ? j : 0) * hd;
            const float4 *kj = reinterpret_cast<const float4 *>(kcache + off);
            const float4 *vj = reinterpret_cast<const float4 *>(vcache + off);
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                kk[u][c] = kj[li + c * lpr];
                vv[u][c] = vj[li + c * lpr];
            }
        }
        float sc[U], mn = m;
#pragma unroll
        for (int u = 0; u < U; u++) {
            float a = 0.0f;
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                a = fmaf(qv[c].x, kk[u][c].x, a);
                a = fmaf(qv[c].y, kk[u][c].y, a);
                a = fmaf(qv[c].z, kk[u][c].z, a);
                a = fmaf(qv[c].w, kk[u][c].w, a);
            }
            for (int o = lpr >> 1; o > 0; o >>= 1)
                a += __shfl_xor_sync(0xffffffffu, a, o);
            sc[u] = j0 + u * stride + sub < npos ? a * scale : -INFINITY;
            mn = fmaxf(mn, sc[u]);
        }
        if (mn == -INFINITY)
            continue; /* no position of this row group in the step */
        const float corr = expf(m - mn); /* 0 while m is still -inf */
        l *= corr;
#pragma unroll
        for (int c = 0; c < CPL; c++) {
            acc[c].x *= corr;
            acc[c].y *= corr;
            acc[c].z *= corr;
            acc[c].w *= corr;
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const float p = expf(sc[u] - mn); /* 0 for masked rows */
            l += p;
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                acc[c].x = fmaf(p, vv[u][c].x, acc[c].x);
                acc[c].y = fmaf(p, vv[u][c].y, acc[c].y);
                acc[c].z = fmaf(p, vv[u][c].z, acc[c].z);
                acc[c].w = fmaf(p, vv[u][c].w, acc[c].w);
            }
        }
        m = mn;
    }
    const int state = warp * rpi + sub;
    if (li == 0) {
        st_m[state] = m;
        st_l[state] = l;
    }
#pragma unroll
    for (int c = 0; c < CPL; c++)
        reinterpret_cast<float4 *>(st_c + size_t(state) * hd)[li + c * lpr] = acc[c];
    __syncthreads();
    float M = -INFINITY;
    for (int k = 0; k < nst; k++)
        M = fmaxf(M, st_m[k]);
    __half *out = ctx + size_t(b) * Kp + h * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float L = 0.0f, c = 0.0f;
        for (int k = 0; k < nst; k++) {
            if (st_m[k] == -INFINITY)
                continue;
            const float f = expf(st_m[k] - M);
            L = fmaf(st_l[k], f, L);
            c = fmaf(st_c[size_t(k) * hd + d], f, c);
        }
        out[d] = to_half_sat(c / L);
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

/* One CTA per (chunk of kArgChunk logits, row): the chunk's largest key
 * goes to keys[b] with a 64-bit atomic max, so keys[b] must be zero before
 * the launch (keys_to_ids zeroes it once read). */
constexpr int kArgThreads = 256;
constexpr int kArgChunk = kArgThreads * 8;

__global__ void argmax_keys_kernel(const float *logits, int V, int v0, unsigned long long *keys,
                                   float *clear) {
    __shared__ unsigned long long best[kArgThreads / 32];
    const int b = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = blockIdx.x * kArgChunk, c1 = min(V, c0 + kArgChunk);
    const float *row = logits + size_t(b) * V;
    float *crow = clear != nullptr ? clear + size_t(b) * V : nullptr;
    unsigned long long k = 0ull;
    const bool vec = (V & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
    if (vec) {
        for (int i = c0 + 4 * int(threadIdx.x); i < c1; i += 4 * kArgThreads) {
            const float4 v = *reinterpret_cast<const float4 *>(row + i);
            const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const unsigned long long c = argmax_key(e[j], uint32_t(v0 + i + j));
                k = c > k ? c : k;
            }
            if (crow != nullptr) /* consumed: the next split-K GEMM adds into it */
                *reinterpret_cast<float4 *>(crow + i) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    } else {
        for (int i = c0 + int(threadIdx.x); i < c1; i += kArgThreads) {
            const unsigned long long c = argmax_key(row[i], uint32_t(v0 + i));
            k = c > k ? c : k;
            if (crow != nullptr)
                crow[i] = 0.0f;
        }
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
        for (int w = 0; w < kArgThreads / 32; w++)
            m = best[w] > m ? best[w] : m;
        atomicMax(keys + b, m);
    }
}

__global__ void keys_to_ids_kernel(unsigned long long *keys, int B, int32_t *ids,
                                   int32_t *out, int ld, const int *step) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B)
        return;
    const int32_t t = int32_t(argmax_index(keys[b]));
    keys[b] = 0ull; /* ready for the next atomic max */
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

/* One thread per packed 32-bit word of nibbles (8 consecutive k, in the
 * packed order k0 k2 k4 k6 k1 k3 k5 k7, each q + 8 with q = hash % 15 - 7)
 * or per scale byte (scales as in synth_int4_f16_kernel). */
__global__ void synth_q4_packed_kernel(uint64_t seed, uint64_t stream, float sigma, int rows,
                                       int cols, int kbs, uint8_t *out) {
    constexpr int kWords = kQ4Rows * 8, kScaleBytes = kQ4Rows * 4;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int tiles = (rows + kQ4Rows - 1) / kQ4Rows;
    if (i >= int64_t(tiles) * kbs * (kWords + kScaleBytes))
        return;
    const int64_t stage = i / (kWords + kScaleBytes);
    const int off = int(i - stage * (kWords + kScaleBytes));
    const int nt = int(stage / kbs), kb = int(stage - int64_t(nt) * kbs);
    uint8_t *st = out + stage * kQ4StageBytes;
    const float unit = sigma * 2.5f / 7.0f;
    if (off < kWords) {
        const int r = off / 8, wd = off % 8, row = nt * kQ4Rows + r;
        const int k0 = kb * 64 + wd * 8;
        uint32_t word = 0x88888888u; /* q = 0 */
        if (row < rows && k0 + 8 <= cols) {
            word = 0;
            for (int k = 0; k < 8; k++) {
                const uint32_t q8 =
                    uint32_t(element_hash(seed, stream, uint64_t(row) * cols + k0 + k) % 15u) + 1u;
                const int slot = (k & 1) ? 4 + k / 2 : k / 2;
                word |= q8 << (4 * slot); /* q + 8 with q in [-7, 7] */
            }
        }
        reinterpret_cast<uint32_t *>(st)[off] = word;
    } else {
        const int sb = off - kWords;
        const int j = sb / 2, byte = sb % 2;
        const int r = j / 2, h = j % 2, row = nt * kQ4Rows + r, blk = kb * 2 + h;
        uint16_t bits = 0;
        if (row < rows && (blk + 1) * 32 <= cols) {
            const uint64_t hs = element_hash(seed, stream ^ 0x5CA1Eull, uint64_t(row) * cols + blk);
            bits = __half_as_ushort(__float2half_rn(
                unit * (0.75f + 0.5f * float(uint32_t(hs >> 40)) * (1.0f / 16777216.0f))));
        }
        st[kQ4Rows * 32 + sb] = byte == 0 ? uint8_t(bits & 0xFF) : uint8_t(bits >> 8);
    }
}

} // namespace

cudaError_t synth_q4_packed_dev(uint64_t seed, uint64_t stream, float sigma, int rows,
                                int cols, int K, uint8_t *out, cudaStream_t s) {
    const int kbs = K / 64, tiles = (rows + kQ4Rows - 1) / kQ4Rows;
    const int64_t n = int64_t(tiles) * kbs * (kQ4Rows * 8 + kQ4Rows * 4);
    synth_q4_packed_kernel<<<blocks_for(n, 256), 256, 0, s>>>(seed, stream, sigma, rows, cols,
                                                              kbs, out);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t add_rmsnorm_rows(float *h, float *part, bool add, const float *w, int B, int dim,
                             int Kp, uint16_t *out, cudaStream_t s) {
    const bool vec = dim % 4 == 0 && Kp % 2 == 0 && dim <= 4 * kNormVec * kNormThreads &&
                     ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(part) |
                       reinterpret_cast<uintptr_t>(w)) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 3) == 0;
    if (vec)
        add_rmsnorm_rows_vec_kernel<<<B, kNormThreads, 0, s>>>(
            h, part, add ? 1 : 0, w, dim, Kp, reinterpret_cast<__half *>(out));
    else
        add_rmsnorm_rows_kernel<<<B, 1024, 0, s>>>(h, part, add ? 1 : 0, w, dim, Kp,
                                                   reinterpret_cast<__half *>(out));
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t rope_kv_batch(float *qkv, int B, int ldq, const int *pos, const float *rope_cos,
                          const float *rope_sin, int heads, int kv_heads, int hd,
                          float *kcache, float *vcache, int layer, int max_seq,
                          cudaStream_t s, int rows, int pf_n, int seq0) {
    if (rows <= 0)
        rows = B;
    const int64_t n = int64_t(rows) * (heads * (hd / 2) + kv_heads * (hd / 2) + kv_heads * hd);
    rope_kv_batch_kernel<<<blocks_for(n, 256), 256, 0, s>>>(qkv, rows, B, ldq, pos, rope_cos,
                                                            rope_sin, heads, kv_heads, hd,
                                                            kcache, vcache, layer, max_seq, pf_n,
                                                            seq0);
    count_launches(1);
    return cudaGetLastError();
}

template <int CPL>
cudaError_t launch_attention(const float *qkv, int rows, int B, int ldq, const int *pos,
                             const float *kcache, const float *vcache, int layer, int heads,
                             int kv_heads, int hd, int max_seq, int Kp, __half *ctx, int lpr,
                             cudaStream_t s) {
    const size_t nst = size_t(kAttWarps) * size_t(32 / lpr);
    const size_t smem = (size_t(hd) * (1 + nst) + 2 * nst) * sizeof(float);
    auto k = attention_batch_kernel<CPL>;
    if (smem > 48 * 1024) {
        const cudaError_t e =
            cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess)
            return e;
    }
    k<<<rows * heads, kAttWarps * 32, smem, s>>>(qkv, B, ldq, pos, kcache, vcache, layer, heads,
                                                 kv_heads, hd, max_seq, Kp, ctx);
    return cudaGetLastError();
}

cudaError_t attention_batch(const float *qkv, int B, int ldq, const int *pos,
                            const float *kcache, const float *vcache, int layer, int heads,
                            int kv_heads, int hd, int max_seq, int Kp, uint16_t *ctx,
                            cudaStream_t s) {
    const int rows = B;
    /* float4 rows over lpr lanes (the largest power of two dividing
     * hd / 4, at most 32), CPL float4 per lane */
    if (hd % 4 != 0 || hd <= 0)
        return cudaErrorInvalidValue;
    int lpr = 32;
    while ((hd / 4) % lpr != 0)
        lpr >>= 1;
    const int cpl = hd / 4 / lpr;
    __half *c16 = reinterpret_cast<__half *>(ctx);
    cudaError_t e;
    switch (cpl) {
    case 1:
        e = launch_attention<1>(qkv, rows, B, ldq, pos, kcache, vcache, layer, heads,
                                kv_heads, hd, max_seq, Kp, c16, lpr, s);
        break;
    case 2:
        e = launch_attention<2>(qkv, rows, B, ldq, pos, kcache, vcache, layer, heads,
                                kv_heads, hd, max_seq, Kp, c16, lpr, s);
        break;
    case 3:
        e = launch_attention<3>(qkv, rows, B, ldq, pos, kcache, vcache, layer, heads,
                                kv_heads, hd, max_seq, Kp, c16, lpr, s);
        break;
    case 4:
        e = launch_attention<4>(qkv, rows, B, ldq, pos, kcache, vcache, layer, heads,
                                kv_heads, hd, max_seq, Kp, c16, lpr, s);
        break;
    default:
        return cudaErrorInvalidValue;
    }
    count_launches(1);
    if (e != cudaSuccess)
        return e;
    if (Kp > heads * hd) {
        const int64_t n = int64_t(rows) * (Kp - heads * hd);
        zero_cols_kernel<<<blocks_for(n, 256), 256, 0, s>>>(c16, rows, heads * hd, Kp);
        count_launches(1);
    }
    return cudaGetLastError();
}

cudaError_t argmax_keys(const float *logits, int B, int V, int v0, unsigned long long *keys,
                        bool clear, cudaStream_t s) {
    const dim3 grid(unsigned((V + kArgChunk - 1) / kArgChunk), unsigned(B));
    argmax_keys_kernel<<<grid, kArgThreads, 0, s>>>(logits, V, v0, keys,
                                                   clear ? const_cast<float *>(logits) : nullptr);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t keys_to_ids(unsigned long long *keys, int B, int32_t *ids, int32_t *out,
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

namespace nut {
namespace {

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct PeerPtrs {
    float *recv[8];
    unsigned *flags[8];
};

__global__ void __launch_bounds__(256)
peer_all_reduce_kernel(const float *x, float *out, int n, PeerPtrs pp, int rank, int world,
                       unsigned *epochs, int *error, uint64_t limit_ns) {
    const int c = blockIdx.x;
    const int per = (n / 4 + kArChunks - 1) / kArChunks; /* float4 per chunk */
    const int f0 = c * per, f1 = min(n / 4, f0 + per);
    __shared__ unsigned epoch_s;
    __shared__ int failed;
    if (threadIdx.x == 0) {
        epoch_s = epochs[c] + 1;
        failed = 0;
    }
    __syncthreads();
    const unsigned e = epoch_s;
    const size_t slot = size_t(e & 1u) * size_t(world) * size_t(n);
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    /* push this rank's chunk into every rank's receive area */
    for (int i = f0 + int(threadIdx.x); i < f1; i += blockDim.x) {
        const float4 v = x4[i];
        for (int q = 0; q < world; q++)
            reinterpret_cast<float4 *>(pp.recv[q] + slot + size_t(rank) * n)[i] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system(); /* the chunk's stores before its flags */
        for (int q = 0; q < world; q++)
            st_release_sys(pp.flags[q] + size_t(rank) * kArChunks + c, e);
    }
    /* wait for chunk c of every rank (thread q polls rank q's flag) */
    if (int(threadIdx.x) < world) {
        const unsigned *f = pp.flags[rank] + size_t(threadIdx.x) * kArChunks + c;
        if (ld_acquire_sys(f) != e) {
            const uint64_t t0 = now_ns();
            while (ld_acquire_sys(f) != e) {
                if (now_ns() - t0 > limit_ns) {
                    atomicExch(&failed, 1);
                    atomicCAS(error, 0, 1);
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!failed) {
        /* read through L2: the peers wrote these lines over NVLink */
        const float *mine = pp.recv[rank] + slot;
        for (int i = f0 + int(threadIdx.x); i < f1; i += blockDim.x) {
            float4 a = __ldcg(reinterpret_cast<const float4 *>(mine) + i);
            for (int q = 1; q < world; q++) {
                const float4 b = __ldcg(reinterpret_cast<const float4 *>(mine + size_t(q) * n) + i);
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
            }
            reinterpret_cast<float4 *>(out)[i] = a;
        }
    }
    if (threadIdx.x == 0)
        epochs[c] = e;
}

} // namespace

cudaError_t peer_all_reduce(const float *x, float *out, int n, float *const *recv,
                            unsigned *const *flags, int rank, int world, unsigned *epochs,
                            int *error, uint64_t limit_ns, cudaStream_t s) {
    if (world < 1 || world > 8 || n % 4 != 0 || rank < 0 || rank >= world)
        return cudaErrorInvalidValue;
    PeerPtrs pp{};
    for (int q = 0; q < world; q++) {
        pp.recv[q] = recv[q];
        pp.flags[q] = flags[q];
    }
    peer_all_reduce_kernel<<<kArChunks, 256, 0, s>>>(x, out, n, pp, rank, world, epochs, error,
                                                     limit_ns);
    count_launches(1);
    return cudaGetLastError();
}

} // namespace nut
