#pragma once
/* Dense row-major fp32 matrix with 64-byte aligned host storage.
 *
 * Same contract as the reference's Matrix (include/tensor.hpp:12-77):
 * move-only, zero dimensions rejected with std::invalid_argument, overflow
 * with std::length_error, at(r, c) row-major access. */
#include <cstddef>
#include <cstdlib>
#include <limits>
#include <new>
#include <stdexcept>

class Matrix {
public:
    static constexpr size_t kAlign = 64;

    Matrix() = default;
    Matrix(size_t rows, size_t cols) : rows_(rows), cols_(cols) {
        if (rows == 0 || cols == 0)
            throw std::invalid_argument("Matrix: zero dimension");
        if (rows > std::numeric_limits<size_t>::max() / cols ||
            rows * cols > std::numeric_limits<size_t>::max() / sizeof(float) -
                              kAlign)
            throw std::length_error("Matrix: dimensions overflow");
        const size_t bytes = (rows * cols * sizeof(float) + kAlign - 1) /
                             kAlign * kAlign;
        data_ = static_cast<float *>(std::aligned_alloc(kAlign, bytes));
        if (data_ == nullptr)
            throw std::bad_alloc();
    }
    ~Matrix() { std::free(data_); }
    Matrix(const Matrix &) = delete;
    Matrix &operator=(const Matrix &) = delete;
    Matrix(Matrix &&o) noexcept : data_(o.data_), rows_(o.rows_), cols_(o.cols_) {
        o.data_ = nullptr;
        o.rows_ = o.cols_ = 0;
    }
    Matrix &operator=(Matrix &&o) noexcept {
        if (this != &o) {
            std::free(data_);
            data_ = o.data_;
            rows_ = o.rows_;
            cols_ = o.cols_;
            o.data_ = nullptr;
            o.rows_ = o.cols_ = 0;
        }
        return *this;
    }

    float *data() { return data_; }
    const float *data() const { return data_; }
    size_t rows() const { return rows_; }
    size_t cols() const { return cols_; }
    size_t size() const { return rows_ * cols_; }
    float &at(size_t r, size_t c) { return data_[r * cols_ + c]; }
    float at(size_t r, size_t c) const { return data_[r * cols_ + c]; }
    void fill(float v) {
        for (size_t i = 0; i < size(); i++)
            data_[i] = v;
    }
    void zero() { fill(0.0f); }

private:
    float *data_ = nullptr;
    size_t rows_ = 0;
    size_t cols_ = 0;
};
