/* Per-phase token-loop kernels over the reference storage layout.
 *
 * One launch per phase of decode_quantized_token (reference
 * src/quant_model.cpp:158-206): rmsnorm-prologue quantised matvecs, RoPE +
 * KV append, GQA attention, SwiGLU, and the final rmsnorm + fp32 lm_head +
 * first-index argmax of the greedy loop (src/generate.cpp:197-201).
 */
#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace nut {
namespace {

constexpr int kMatvecThreads = 256;

/* The staged input vector is kept in shared memory in 16-byte granules,
 * swizzled per 32-float block so that lanes reading granule g of
 * consecutive blocks hit distinct banks. */
__device__ __forceinline__ int swz(int i) {
    const int b = i >> 5, g = (i >> 2) & 7;
    return (b << 5) | ((g ^ (b & 7)) << 2) | (i & 3);
}

__device__ __forceinline__ float nib(uint32_t w, int k) {
    return float(int32_t(w << (28 - 4 * k)) >> 28);
}

__device__ __forceinline__ float byte_s8(uint32_t w, int k) {
    return float(int32_t(w << (24 - 8 * k)) >> 24);
}

/* Sum over one 32-weight block: 16 packed bytes (INT4) or 32 bytes (INT8)
 * against the swizzled x block b. */
template <int TYPE>
__device__ __forceinline__ float block_dot(const uint8_t *__restrict__ w,
                                           const float4 *__restrict__ xs4,
                                           int b) {
    float acc = 0.0f;
    const int sw = b & 7;
    if (TYPE == 1) {
        const uint4 p = __ldg(reinterpret_cast<const uint4 *>(w));
        const uint32_t words[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float4 xa = xs4[b * 8 + ((2 * j) ^ sw)];
            const float4 xb = xs4[b * 8 + ((2 * j + 1) ^ sw)];
            acc = fmaf(nib(words[j], 0), xa.x, acc);
            acc = fmaf(nib(words[j], 1), xa.y, acc);
            acc = fmaf(nib(words[j], 2), xa.z, acc);
            acc = fmaf(nib(words[j], 3), xa.w, acc);
            acc = fmaf(nib(words[j], 4), xb.x, acc);
            acc = fmaf(nib(words[j], 5), xb.y, acc);
            acc = fmaf(nib(words[j], 6), xb.z, acc);
            acc = fmaf(nib(words[j], 7), xb.w, acc);
        }
    } else {
        const uint4 p0 = __ldg(reinterpret_cast<const uint4 *>(w));
        const uint4 p1 = __ldg(reinterpret_cast<const uint4 *>(w) + 1);
        const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w,
                                   p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 x = xs4[b * 8 + (j ^ sw)];
            acc = fmaf(byte_s8(words[j], 0), x.x, acc);
            acc = fmaf(byte_s8(words[j], 1), x.y, acc);
            acc = fmaf(byte_s8(words[j], 2), x.z, acc);
            acc = fmaf(byte_s8(words[j], 3), x.w, acc);
        }
    }
    return acc;
}

__device__ __forceinline__ int qvalue(int type, const uint8_t *data, int64_t i) {
    if (type == 0)
        return int(int8_t(data[i]));
    const unsigned n = (i & 1) ? (data[i >> 1] >> 4) : (data[i >> 1] & 0xfu);
    return n >= 8 ? int(n) - 16 : int(n);
}

template <int TYPE>
__global__ void __launch_bounds__(kMatvecThreads)
qmatvec_kernel(QSegs segs, const float *__restrict__ src,
               const float *__restrict__ norm) {
    extern __shared__ float4 xs4[];
    __shared__ float red[32];
    float *xs = reinterpret_cast<float *>(xs4);
    const int K = segs.cols;
    float scale = 1.0f;
    if (norm != nullptr) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const float v = src[i];
            ss = fmaf(v, v, ss);
        }
        const float total = block_sum(ss, red);
        scale = 1.0f / sqrtf(total / float(K) + kEps);
    }
    for (int i = threadIdx.x; i < K; i += blockDim.x) {
        float v = src[i];
        if (norm != nullptr)
            v = v * scale * norm[i];
        xs[swz(i)] = v;
    }
    __syncthreads();

    int total_rows = 0;
    for (int s = 0; s < segs.count; s++)
        total_rows += segs.seg[s].rows;
    const bool aligned = (K % kBlock) == 0;
    if (!aligned) {
        /* Blocks span rows (cols % 32 != 0): one thread per row over the
         * flattened blocks, double accumulation as the reference's scalar
         * path (src/quant.cpp:289-317). */
        for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < total_rows;
             r += gridDim.x * blockDim.x) {
            int s = 0, row = r;
            while (row >= segs.seg[s].rows) {
                row -= segs.seg[s].rows;
                s++;
            }
            const QSeg &g = segs.seg[s];
            double sum = 0.0;
            const int64_t begin = int64_t(row) * K;
            for (int c = 0; c < K; c++) {
                const int64_t i = begin + c;
                const float sc = half_bits_to_float(g.scales[i / kBlock]);
                sum += double(float(qvalue(TYPE, g.data, i)) * sc) *
                       double(xs[swz(c)]);
            }
            const float y = float(sum);
            g.out[row] = g.accumulate ? g.out[row] + y : y;
        }
        return;
    }

    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    const int nblocks = K / kBlock;
    const int row_bytes = TYPE == 1 ? K / 2 : K;
    const int blk_bytes = TYPE == 1 ? 16 : 32;
    for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < total_rows;
         r += gridDim.x * warps) {
        int s = 0, row = r;
        while (row >= segs.seg[s].rows) {
            row -= segs.seg[s].rows;
            s++;
        }
        const QSeg &g = segs.seg[s];
        const uint8_t *wrow = g.data + size_t(row) * row_bytes;
        const uint16_t *srow = g.scales + size_t(row) * nblocks;
        float acc = 0.0f;
        for (int b = lane; b < nblocks; b += 32)
            acc = fmaf(half_bits_to_float(srow[b]),
                       block_dot<TYPE>(wrow + b * blk_bytes, xs4, b), acc);
        acc = warp_sum(acc);
        if (lane == 0)
            g.out[row] = g.accumulate ? g.out[row] + acc : acc;
    }
}

__global__ void embed_kernel(const float *__restrict__ embeddings, int dim,
                             int vocab, int token,
                             unsigned long long *argmax_key,
                             int32_t *id_slot, float *__restrict__ hidden) {
    __shared__ int tok;
    if (threadIdx.x == 0) {
        int t = token;
        if (t < 0) {
            const uint32_t a = argmax_index(*argmax_key);
            /* an argmax key is always set before a device-fed token is
             * read; the bound keeps a stale key from indexing past the
             * table */
            t = a < uint32_t(vocab) ? int(a) : 0;
            if (id_slot != nullptr)
                *id_slot = t;
        }
        tok = t;
    }
    __syncthreads();
    const float *row = embeddings + size_t(tok) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        hidden[i] = row[i];
}

/* Interleaved-pair RoPE (src/quant_model.cpp:26-37) on q and k with the
 * host-computed fp32 cos/sin table, then KVCache::store of k and v
 * (src/kvcache.cpp:216-229) at `position`. */
__global__ void rope_store_kernel(float *__restrict__ q,
                                  const float *__restrict__ k,
                                  const float *__restrict__ v,
                                  float *__restrict__ kcache,
                                  float *__restrict__ vcache,
                                  const float *__restrict__ rope_cos,
                                  const float *__restrict__ rope_sin,
                                  int position, int layer, int heads,
                                  int kv_heads, int hd, int max_seq) {
    const int half = hd / 2;
    const int nq = heads * half, nk = kv_heads * half, nv = kv_heads * hd;
    const float *cs = rope_cos + size_t(position) * half;
    const float *sn = rope_sin + size_t(position) * half;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nq + nk + nv;
         i += gridDim.x * blockDim.x) {
        if (i < nq) {
            const int h = i / half, j = i % half;
            float *p = q + h * hd + 2 * j;
            const float e = p[0], o = p[1];
            p[0] = e * cs[j] - o * sn[j];
            p[1] = e * sn[j] + o * cs[j];
        } else if (i < nq + nk) {
            const int t = i - nq, h = t / half, j = t % half;
            const float e = k[h * hd + 2 * j], o = k[h * hd + 2 * j + 1];
            float *dst = kcache +
                         ((size_t(layer) * kv_heads + h) * max_seq + position) * hd +
                         2 * j;
            dst[0] = e * cs[j] - o * sn[j];
            dst[1] = e * sn[j] + o * cs[j];
        } else {
            const int t = i - nq - nk, h = t / hd, d = t % hd;
            vcache[((size_t(layer) * kv_heads + h) * max_seq + position) * hd + d] =
                v[t];
        }
    }
}

/* GQA attention for one query head per CTA over positions 0..position
 * (attention_step, src/quant_model.cpp:68-105): scores scaled by
 * 1/sqrt(head_dim), max-shifted exp, weights score/total, context. */
__global__ void attention_kernel(const float *__restrict__ q,
                                 const float *__restrict__ kcache,
                                 const float *__restrict__ vcache,
                                 float *__restrict__ ctx, int position,
                                 int layer, int heads, int kv_heads, int hd,
                                 int max_seq) {
    extern __shared__ float sm[];
    __shared__ float red[32];
    float *qs = sm;
    float *scores = sm + hd;
    const int h = blockIdx.x;
    const int kvh = h / (heads / kv_heads);
    const size_t base = (size_t(layer) * kv_heads + kvh) * size_t(max_seq) * hd;
    const int n = position + 1;
    for (int d = threadIdx.x; d < hd; d += blockDim.x)
        qs[d] = q[h * hd + d];
    __syncthreads();
    const float scale = 1.0f / sqrtf(float(hd));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    for (int p = warp; p < n; p += warps) {
        const float *key = kcache + base + size_t(p) * hd;
        float dot = 0.0f;
        for (int d = lane; d < hd; d += 32)
            dot = fmaf(qs[d], key[d], dot);
        dot = warp_sum(dot);
        if (lane == 0)
            scores[p] = dot * scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int p = threadIdx.x; p < n; p += blockDim.x)
        m = fmaxf(m, scores[p]);
    m = block_max(m, red);
    float local = 0.0f;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        const float e = expf(scores[p] - m);
        scores[p] = e;
        local += e;
    }
    const float total = block_sum(local, red);
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float acc = 0.0f;
        for (int p = 0; p < n; p++)
            acc = fmaf(scores[p] / total,
                       vcache[base + size_t(p) * hd + d], acc);
        ctx[h * hd + d] = acc;
    }
}

/* gate[i] = silu(gate[i]) * up[i] (src/quant_model.cpp:197-198,
 * silu src/ops.cpp:136-138). */
__global__ void swiglu_kernel(float *__restrict__ gate,
                              const float *__restrict__ up, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += gridDim.x * blockDim.x) {
        const float g = gate[i];
        gate[i] = g / (1.0f + expf(-g)) * up[i];
    }
}

/* logits = W rmsnorm(hidden, final_norm); argmax into *key by atomicMax. */
__global__ void __launch_bounds__(256)
lmhead_kernel(const float *__restrict__ hidden,
              const float *__restrict__ final_norm,
              const float *__restrict__ weights, int vocab, int dim,
              float *__restrict__ logits, unsigned long long *key) {
    extern __shared__ float4 xs4f[];
    __shared__ float red[32];
    __shared__ unsigned long long best_key[8];
    float *xs = reinterpret_cast<float *>(xs4f);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        ss = fmaf(hidden[i], hidden[i], ss);
    const float total = block_sum(ss, red);
    const float scale = 1.0f / sqrtf(total / float(dim) + kEps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        xs[i] = hidden[i] * scale * final_norm[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    unsigned long long mine = 0ull;
    const bool vec = (dim % 4) == 0;
    for (int r = blockIdx.x * warps + warp; r < vocab; r += gridDim.x * warps) {
        const float *row = weights + size_t(r) * dim;
        float acc = 0.0f;
        if (vec) {
            const float4 *row4 = reinterpret_cast<const float4 *>(row);
            for (int g = lane; g < dim / 4; g += 32) {
                const float4 w = __ldg(row4 + g);
                const float4 x = xs4f[g];
                acc = fmaf(w.x, x.x, acc);
                acc = fmaf(w.y, x.y, acc);
                acc = fmaf(w.z, x.z, acc);
                acc = fmaf(w.w, x.w, acc);
            }
        } else {
            for (int c = lane; c < dim; c += 32)
                acc = fmaf(row[c], xs[c], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            if (logits != nullptr)
                logits[r] = acc;
            const unsigned long long k = argmax_key(acc, uint32_t(r));
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
            atomicMax(key, b);
    }
}

int sm_count() {
    static int count = 0;
    if (count == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
        if (count <= 0)
            count = 148;
    }
    return count;
}

} // namespace

void launch_qmatvec(const QSegs &segs, const float *src, const float *norm,
                    cudaStream_t stream) {
    int rows = 0;
    for (int s = 0; s < segs.count; s++)
        rows += segs.seg[s].rows;
    const size_t smem = size_t((segs.cols + 31) / 32) * 32 * sizeof(float);
    const bool aligned = segs.cols % kBlock == 0;
    const int per_cta = aligned ? kMatvecThreads / 32 : kMatvecThreads;
    int grid = (rows + per_cta - 1) / per_cta;
    grid = grid < 4 * sm_count() ? grid : 4 * sm_count();
    if (segs.type == 1) {
        cudaFuncSetAttribute(qmatvec_kernel<1>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        qmatvec_kernel<1><<<grid, kMatvecThreads, smem, stream>>>(segs, src, norm);
        count_launches(1);
    } else {
        cudaFuncSetAttribute(qmatvec_kernel<0>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        qmatvec_kernel<0><<<grid, kMatvecThreads, smem, stream>>>(segs, src, norm);
        count_launches(1);
    }
}

void launch_embed(const float *embeddings, int dim, int vocab, int token,
                  unsigned long long *argmax_key, int32_t *id_slot,
                  float *hidden, cudaStream_t stream) {
    embed_kernel<<<1, 256, 0, stream>>>(embeddings, dim, vocab, token,
                                        argmax_key, id_slot, hidden);
    count_launches(1);
}

void launch_rope_store(float *q, const float *k, const float *v, float *kcache,
                       float *vcache, const float *rope_cos,
                       const float *rope_sin, int position, int layer,
                       int heads, int kv_heads, int head_dim, int max_seq,
                       cudaStream_t stream) {
    const int work = heads * head_dim / 2 + kv_heads * head_dim / 2 +
                     kv_heads * head_dim;
    const int grid = (work + 255) / 256;
    rope_store_kernel<<<grid, 256, 0, stream>>>(q, k, v, kcache, vcache,
                                                rope_cos, rope_sin, position,
                                                layer, heads, kv_heads,
                                                head_dim, max_seq);
    count_launches(1);
}

void launch_attention(const float *q, const float *kcache, const float *vcache,
                      float *ctx, int position, int layer, int heads,
                      int kv_heads, int head_dim, int max_seq,
                      cudaStream_t stream) {
    const size_t smem = sizeof(float) * size_t(head_dim + position + 1);
    cudaFuncSetAttribute(attention_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    attention_kernel<<<heads, 128, smem, stream>>>(q, kcache, vcache, ctx,
                                                   position, layer, heads,
                                                   kv_heads, head_dim, max_seq);
    count_launches(1);
}

void launch_swiglu(float *gate, const float *up, int n, cudaStream_t stream) {
    swiglu_kernel<<<(n + 255) / 256, 256, 0, stream>>>(gate, up, n);
    count_launches(1);
}

void launch_lmhead(const float *hidden, const float *final_norm,
                   const float *weights, int vocab, int dim, float *logits,
                   unsigned long long *argmax_key, cudaStream_t stream) {
    const size_t smem = size_t((dim + 3) / 4) * 16;
    cudaFuncSetAttribute(lmhead_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    int grid = (vocab + 7) / 8;
    grid = grid < 4 * sm_count() ? grid : 4 * sm_count();
    lmhead_kernel<<<grid, 256, smem, stream>>>(hidden, final_norm, weights,
                                               vocab, dim, logits, argmax_key);
    count_launches(1);
}

} // namespace nut
