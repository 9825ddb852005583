#pragma once
/* Per-block symmetric INT8/INT4 quantised matrices — host side of the
 * drop-in for the reference's include/quant.hpp:9-59.
 *
 * Storage is the reference's, byte for byte: flattened row-major blocks of
 * 32 weights, one fp16 scale (as uint16_t bits) per block, INT8 one byte per
 * weight, INT4 two's-complement nibbles with the even flattened index in the
 * low nibble.  matvec_quantized[_threaded] runs on the GPU through the
 * C-ABI; the device copy of the matrix is made on first use and kept. */
#include <cstddef>
#include <cstdint>
#include <memory>
#include <vector>

#include "tensor.hpp"

enum class QuantType {
    int8,
    int4,
};

struct nut_qmatrix;

class QuantizedMatrix {
public:
    static QuantizedMatrix quantize(const Matrix &source, QuantType type,
                                    size_t block_size = 32);
    static QuantizedMatrix quantize(const float *source, size_t rows,
                                    size_t cols, QuantType type,
                                    size_t block_size = 32);
    /* Adopts already-quantised bytes (e.g. read back from a device). */
    static QuantizedMatrix from_storage(size_t rows, size_t cols, QuantType type,
                                        std::vector<uint8_t> data,
                                        std::vector<uint16_t> scales);

    size_t rows() const { return rows_; }
    size_t cols() const { return cols_; }
    size_t size() const { return rows_ * cols_; }
    size_t block_size() const { return block_size_; }
    size_t blocks() const { return scales_.size(); }
    QuantType type() const { return type_; }
    size_t storage_bytes() const;
    uint8_t packed_byte(size_t index) const;

    float value(size_t row, size_t column) const;
    float error_bound(size_t row, size_t column) const;

    /* Raw storage, for uploading to the device. */
    const std::vector<uint8_t> &data() const { return data_; }
    const std::vector<uint16_t> &scales() const { return scales_; }

    /* Device mirror (created on first use on the current device). */
    nut_qmatrix *device_handle() const;

private:
    QuantizedMatrix(size_t rows, size_t cols, size_t block_size, QuantType type);
    int quantized_value(size_t index) const;
    float scale(size_t block) const;

    size_t rows_;
    size_t cols_;
    size_t block_size_;
    QuantType type_;
    std::vector<uint8_t> data_;
    std::vector<uint16_t> scales_;
    mutable std::shared_ptr<nut_qmatrix> device_;
};

Matrix dequantize(const QuantizedMatrix &source);
void matvec_quantized(const QuantizedMatrix &matrix, const float *vector,
                      float *output);
void matvec_quantized_threaded(const QuantizedMatrix &matrix,
                               const float *vector, float *output,
                               size_t thread_count);

/* fp16 codec of the quantiser (scales are stored as fp16 bits). */
uint16_t quant_scale_to_half(float value);
float quant_half_to_float(uint16_t value);
