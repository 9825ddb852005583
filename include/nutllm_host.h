/* nutllm_host.h — C entry points of libnutllm.so, the C++17 host library
 * (load-time quantiser and seeded synthetic inputs).  Status codes are the
 * nut_status values of nutllm_cuda.h. */
#ifndef NUTLLM_HOST_H
#define NUTLLM_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Message of the calling thread's last host-library failure. */
const char *nut_host_last_error(void);

/* QuantizedMatrix::quantize (reference src/quant.cpp:154-197) into caller
 * buffers: data holds rows*cols (INT8) or (rows*cols+1)/2 (INT4) bytes,
 * scales (rows*cols+31)/32 fp16 bit patterns.  type: 0 INT8, 1 INT4. */
int nut_host_quantize(const float *source, int64_t rows, int64_t cols,
                      int32_t type, uint8_t *data, uint16_t *scales);

/* fp16 encoding of one positive scale as the quantiser rounds it. */
int nut_host_scale_to_half(float value, uint16_t *bits);

/* Seeded synthetic inputs (documented in nutllm_b200/host/synth.cpp). */
void nut_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out,
                      size_t n);
void nut_synth_tokens(uint64_t seed, uint64_t stream, int lo, int hi, int *out,
                      size_t n);

#ifdef __cplusplus
}
#endif
#endif /* NUTLLM_HOST_H */
