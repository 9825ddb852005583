/* C entry points of the host library (include/nutllm_host.h). */
#include <cstring>
#include <stdexcept>
#include <string>

#include "../../include/nutllm_cuda.h"
#include "../../include/nutllm_host.h"
#include "quant.hpp"

namespace {

thread_local std::string g_error;

template <typename F> int guarded(F &&body) {
    try {
        body();
        return NUT_OK;
    } catch (const std::invalid_argument &e) {
        g_error = e.what();
        return NUT_INVALID_ARGUMENT;
    } catch (const std::out_of_range &e) {
        g_error = e.what();
        return NUT_OUT_OF_RANGE;
    } catch (const std::length_error &e) {
        g_error = e.what();
        return NUT_LENGTH_ERROR;
    } catch (const std::range_error &e) {
        g_error = e.what();
        return NUT_RANGE_ERROR;
    } catch (const std::exception &e) {
        g_error = e.what();
        return NUT_RUNTIME_ERROR;
    }
}

} // namespace

extern "C" {

const char *nut_host_last_error(void) { return g_error.c_str(); }

int nut_host_quantize(const float *source, int64_t rows, int64_t cols,
                      int32_t type, uint8_t *data, uint16_t *scales) {
    return guarded([&] {
        if (type != 0 && type != 1)
            throw std::invalid_argument("quantize: unknown type");
        if (rows <= 0 || cols <= 0)
            throw std::invalid_argument("quantize: invalid dimensions");
        if (data == nullptr || scales == nullptr)
            throw std::invalid_argument("quantize: null output");
        const QuantizedMatrix m = QuantizedMatrix::quantize(
            source, size_t(rows), size_t(cols),
            type == 0 ? QuantType::int8 : QuantType::int4);
        std::memcpy(data, m.data().data(), m.data().size());
        std::memcpy(scales, m.scales().data(), m.scales().size() * 2);
    });
}

int nut_host_scale_to_half(float value, uint16_t *bits) {
    return guarded([&] { *bits = quant_scale_to_half(value); });
}

} // extern "C"
