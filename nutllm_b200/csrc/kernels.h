#pragma once
/* Host-side launchers for the token-loop kernels (compiled by nvcc into
 * libnutcuda.so; not part of the C ABI). */
#include <cstdint>
#include <cuda_runtime.h>

#include <string>

namespace nut {

/* Sets the calling thread's message returned by nut_last_error(). */
void set_last_error(const std::string &message);

/* Adds n to the process-wide count of kernels this library has launched
 * (read through nut_launch_count). */
void count_launches(unsigned n);
/* The counter itself, and a correction for kernels that were captured
 * into a graph rather than launched (their replays count them instead). */
uint64_t launches_so_far();
void uncount_launches(uint64_t n);

/* fp32 products in the reference build's order (fp32_ops.cu):
 * C[M][N] = A[M][K] B[K][N] (fused, k-sequential) and y = W x (unfused,
 * column-sequential). */
cudaError_t matmul_f32(const float *A, const float *B, float *C, int M, int K, int N,
                       cudaStream_t s);
/* fp32-weight decode helpers (fp32_ops.cu): one-vector rmsnorm
 * (eps 1e-5) and h += y. */
cudaError_t rmsnorm_vec(const float *x, const float *w, float *out, int n, cudaStream_t s);
cudaError_t add_vec(float *h, const float *y, int n, cudaStream_t s);
cudaError_t matvec_f32(const float *W, const float *x, float *y, int rows, int cols,
                       cudaStream_t s);

/* One quantised matrix in the reference storage layout on the device. */
struct DevQMatrix {
    uint8_t *data = nullptr;
    uint16_t *scales = nullptr; /* fp16 bits, one per 32-weight block */
    int64_t rows = 0, cols = 0;
    int type = 0; /* 0 int8, 1 int4 */
    size_t data_bytes() const {
        const int64_t n = rows * cols;
        return size_t(type == 0 ? n : (n + 1) / 2);
    }
    size_t scale_count() const { return size_t((rows * cols + 31) / 32); }
};

/* Output segment of a multi-matrix product sharing one input vector. */
struct QSeg {
    const uint8_t *data;
    const uint16_t *scales;
    int rows;
    float *out;
    int accumulate; /* out[r] += y[r] (residual) instead of out[r] = y[r] */
};

constexpr int kMaxSegs = 3;

struct QSegs {
    QSeg seg[kMaxSegs];
    int count;
    int cols;
    int type;
};

/* y = Q x for up to three matrices sharing x (cols columns).  With norm
 * non-null, x = rmsnorm(src, norm) computed by each CTA first. */
void launch_qmatvec(const QSegs &segs, const float *src, const float *norm,
                    cudaStream_t stream);

void launch_embed(const float *embeddings, int dim, int vocab, int token,
                  unsigned long long *argmax_key, int32_t *id_slot,
                  float *hidden, cudaStream_t stream);

void launch_rope_store(float *q, const float *k, const float *v, float *kcache,
                       float *vcache, const float *rope_cos,
                       const float *rope_sin, int position, int layer,
                       int heads, int kv_heads, int head_dim, int max_seq,
                       cudaStream_t stream);

void launch_attention(const float *q, const float *kcache, const float *vcache,
                      float *ctx, int position, int layer, int heads,
                      int kv_heads, int head_dim, int max_seq,
                      cudaStream_t stream);

void launch_swiglu(float *gate, const float *up, int n, cudaStream_t stream);

void launch_lmhead(const float *hidden, const float *final_norm,
                   const float *weights, int vocab, int dim, float *logits,
                   unsigned long long *argmax_key, cudaStream_t stream);

} // namespace nut
