/* Host quantiser and QuantizedMatrix accessors.
 *
 * A from-scratch restatement of QuantizedMatrix::quantize and its fp16 codec
 * (reference src/quant.cpp:23-56, 154-197); its output bytes and scales are
 * checked bit-exact against the reference by the test suite.  The fp16
 * encoder works on the float's bit fields rather than frexp/lround, with
 * the same rounding: the 13 dropped mantissa bits round half away from zero
 * (the value is positive, so "add half, truncate"), carrying into the
 * exponent; scales below 2^-14 become fp16 subnormals round(v * 2^24)
 * clamped to [1, 1023].  Large matrices are quantised by several threads,
 * each over whole blocks, so the result does not depend on the count. */
#include "quant.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <thread>

#include "device.hpp"

namespace {

/* rows x cols, or invalid_argument when either is zero or the product
 * does not fit in size_t. */
size_t element_count(size_t rows, size_t cols) {
    size_t n = 0;
    const bool wraps = __builtin_mul_overflow(rows, cols, &n);
    if (wraps || n == 0)
        throw std::invalid_argument("quantize: invalid dimensions");
    return n;
}

/* Largest quantised magnitude of a type: 2^(bits-1) - 1. */
constexpr int type_limit(QuantType type) { return type == QuantType::int8 ? 127 : 7; }

uint32_t float_bits(float v) {
    uint32_t b;
    std::memcpy(&b, &v, 4);
    return b;
}

template <typename F> void for_block_ranges(size_t blocks, F &&body) {
    const size_t hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t threads = std::min<size_t>(hw, std::max<size_t>(1, blocks >> 12));
    if (threads <= 1) {
        body(size_t(0), blocks);
        return;
    }
    std::vector<std::thread> pool;
    std::vector<std::exception_ptr> errors(threads);
    for (size_t t = 0; t < threads; t++)
        pool.emplace_back([&, t] {
            try {
                body(blocks * t / threads, blocks * (t + 1) / threads);
            } catch (...) {
                errors[t] = std::current_exception();
            }
        });
    for (auto &th : pool)
        th.join();
    for (auto &e : errors)
        if (e)
            std::rethrow_exception(e); /* first failing range, in order */
}

} // namespace

uint16_t quant_scale_to_half(float value) {
    if (!(value > 0.0f) || !std::isfinite(value))
        throw std::invalid_argument("quantize: scale must be finite positive");
    if (value > 65504.0f)
        throw std::range_error("quantize: scale exceeds fp16");
    const uint32_t bits = float_bits(value);
    const int biased = int(bits >> 23);         /* sign bit is 0 */
    const uint32_t frac = bits & 0x7fffffu;
    if (biased < 127 - 14) {                     /* below 2^-14: subnormal */
        const uint64_t significand = biased == 0 ? frac : (frac | 0x800000u);
        const int exponent = biased == 0 ? -126 : biased - 127;
        /* v * 2^24 = significand * 2^(exponent + 1) with exponent + 1 < 0 */
        const int shift = -(exponent + 1);
        uint64_t m = shift >= 64 ? 0 : (significand + (uint64_t(1) << (shift - 1))) >> shift;
        m = std::clamp<uint64_t>(m, 1, 1023);
        return uint16_t(m);
    }
    int exponent = biased - 127;
    uint32_t mantissa = (frac + 0x1000u) >> 13;
    if (mantissa == 1024) {
        mantissa = 0;
        exponent++;
    }
    if (exponent > 15)
        throw std::range_error("quantize: rounded scale exceeds fp16");
    return uint16_t(((exponent + 15) << 10) | mantissa);
}

float quant_half_to_float(uint16_t value) {
    const unsigned exponent = (value >> 10) & 0x1f;
    const unsigned mantissa = value & 0x3ff;
    if (exponent == 0)
        return std::ldexp(float(mantissa), -24);
    return std::ldexp(1.0f + float(mantissa) / 1024.0f, int(exponent) - 15);
}

QuantizedMatrix::QuantizedMatrix(size_t rows, size_t cols, size_t block_size,
                                 QuantType type)
    : rows_(rows), cols_(cols), block_size_(block_size), type_(type) {
    const size_t n = element_count(rows, cols);
    if (block_size == 0)
        throw std::invalid_argument("quantize: zero block size");
    /* a partial last block still gets a scale: ceil(n / block_size), whose
     * rounded-up numerator must itself fit in size_t */
    size_t padded = 0;
    if (__builtin_add_overflow(n, block_size - 1, &padded))
        throw std::length_error("quantize: block count overflow");
    const size_t blocks = padded / block_size;
    /* int8: one byte per element; int4: two elements per byte, low first */
    const size_t bytes = type == QuantType::int8 ? n : n / 2 + (n & 1);
    scales_.assign(blocks, 0);
    data_.assign(bytes, 0);
}

QuantizedMatrix QuantizedMatrix::quantize(const Matrix &source, QuantType type,
                                          size_t block_size) {
    return quantize(source.data(), source.rows(), source.cols(), type,
                    block_size);
}

QuantizedMatrix QuantizedMatrix::quantize(const float *source, size_t rows,
                                          size_t cols, QuantType type,
                                          size_t block_size) {
    if (source == nullptr)
        throw std::invalid_argument("quantize: null source");
    QuantizedMatrix out(rows, cols, block_size, type);
    const int limit = type_limit(type);
    const size_t n = out.size();
    uint8_t *data = out.data_.data();
    uint16_t *scales = out.scales_.data();
    for_block_ranges(out.blocks(), [&](size_t first, size_t last) {
        for (size_t b = first; b < last; b++) {
            const size_t begin = b * block_size;
            const size_t end = std::min(begin + block_size, n);
            float peak = 0.0f;
            for (size_t i = begin; i < end; i++) {
                if (!std::isfinite(source[i]))
                    throw std::invalid_argument(
                        "quantize: non-finite source weight");
                peak = std::max(peak, std::fabs(source[i]));
            }
            scales[b] = quant_scale_to_half(
                peak == 0.0f ? std::ldexp(1.0f, -24) : peak / float(limit));
            const float stored = quant_half_to_float(scales[b]);
            for (size_t i = begin; i < end; i++) {
                const long q = std::clamp<long>(std::lround(source[i] / stored),
                                                -limit, limit);
                if (type == QuantType::int8) {
                    data[i] = uint8_t(unsigned(q) & 0xffu);
                } else {
                    const uint8_t nibble = uint8_t(q) & 0x0f;
                    /* a block of even size never shares a byte with its
                     * neighbour, so ranges of whole blocks write disjoint
                     * bytes when block_size is even */
                    uint8_t &byte = data[i / 2];
                    byte = i % 2 == 0 ? uint8_t((byte & 0xf0) | nibble)
                                      : uint8_t((byte & 0x0f) | (nibble << 4));
                }
            }
        }
    });
    return out;
}

QuantizedMatrix QuantizedMatrix::from_storage(size_t rows, size_t cols,
                                              QuantType type,
                                              std::vector<uint8_t> data,
                                              std::vector<uint16_t> scales) {
    QuantizedMatrix out(rows, cols, 32, type);
    if (data.size() != out.data_.size() || scales.size() != out.scales_.size())
        throw std::invalid_argument("quantized matrix: storage size mismatch");
    out.data_ = std::move(data);
    out.scales_ = std::move(scales);
    return out;
}

namespace {

/* Flat index of (row, column) in a rows x cols matrix, or out_of_range. */
size_t flat_index(size_t rows, size_t cols, size_t row, size_t column) {
    if (!(row < rows && column < cols))
        throw std::out_of_range("quantized matrix: index out of range");
    return row * cols + column;
}

/* Signed value of a two's-complement field of `bits` bits. */
int sign_extend(unsigned field, int bits) {
    const unsigned top = 1u << (bits - 1);
    return int(field ^ top) - int(top);
}

} // namespace

int QuantizedMatrix::quantized_value(size_t index) const {
    if (!(index < size()))
        throw std::out_of_range("quantized matrix: index out of range");
    if (type_ == QuantType::int4) {
        /* element 2i is the low nibble of byte i, element 2i+1 the high */
        const unsigned byte = data_[index >> 1];
        return sign_extend((byte >> (4 * (index & 1))) & 0x0fu, 4);
    }
    return sign_extend(data_[index], 8);
}

float QuantizedMatrix::scale(size_t block) const {
    if (!(block < scales_.size()))
        throw std::out_of_range("quantized matrix: block out of range");
    return quant_half_to_float(scales_[block]);
}

float QuantizedMatrix::value(size_t row, size_t column) const {
    const size_t i = flat_index(rows_, cols_, row, column);
    const float step = scale(i / block_size_);
    return float(quantized_value(i)) * step;
}

/* The reference's per-element bound (src/quant.cpp:224-233): half a
 * quantisation step, plus (limit + 1/2) times the larger of the fp16
 * scale's relative rounding (scale / 2047) and half an fp16 subnormal
 * step (2^-25). */
float QuantizedMatrix::error_bound(size_t row, size_t column) const {
    const size_t i = flat_index(rows_, cols_, row, column);
    const float step = scale(i / block_size_);
    const float scale_rounding = std::max(step / 2047.0f, 0x1p-25f);
    const float reach = float(type_limit(type_)) + 0.5f;
    return 0.5f * step + reach * scale_rounding;
}

size_t QuantizedMatrix::storage_bytes() const {
    size_t scale_bytes = 0, total = 0;
    if (__builtin_mul_overflow(scales_.size(), sizeof(uint16_t), &scale_bytes) ||
        __builtin_add_overflow(scale_bytes, data_.size(), &total))
        throw std::overflow_error("quantized matrix: storage size overflow");
    return total;
}

uint8_t QuantizedMatrix::packed_byte(size_t index) const {
    const bool packed = type_ == QuantType::int4;
    if (!packed || !(index < data_.size()))
        throw std::out_of_range("quantized matrix: packed byte out of range");
    return data_[index];
}

Matrix dequantize(const QuantizedMatrix &source) {
    Matrix result(source.rows(), source.cols());
    /* one pass over the flat row-major storage */
    float *out = result.data();
    const size_t cols = source.cols();
    for (size_t i = 0, n = source.size(); i < n; i++)
        out[i] = source.value(i / cols, i % cols);
    return result;
}

nut_qmatrix *QuantizedMatrix::device_handle() const {
    if (!device_)
        device_ = nutdev::upload_qmatrix(*this);
    return device_.get();
}

void matvec_quantized(const QuantizedMatrix &matrix, const float *vector,
                      float *output) {
    matvec_quantized_threaded(matrix, vector, output, 1);
}

/* GPU quantised matvec with host buffers.  thread_count keeps the
 * reference's contract (zero rejected) and is otherwise unused: the GPU grid
 * replaces the CPU row split. */
void matvec_quantized_threaded(const QuantizedMatrix &matrix,
                               const float *vector, float *output,
                               size_t thread_count) {
    if (vector == nullptr || output == nullptr)
        throw std::invalid_argument("quantized matvec: null pointer");
    if (thread_count == 0)
        throw std::invalid_argument("quantized matvec: zero threads");
    nutdev::check(nut_qmatvec(matrix.device_handle(), vector, output));
}
