#include "device.hpp"

#include <cstdlib>
#include <stdexcept>
#include <string>

#include "quant.hpp"

namespace nutdev {

namespace {
int g_device = -1;
}

void check(nut_status status) {
    if (status == NUT_OK)
        return;
    const std::string message = nut_last_error();
    switch (status) {
    case NUT_INVALID_ARGUMENT:
        throw std::invalid_argument(message);
    case NUT_OUT_OF_RANGE:
        throw std::out_of_range(message);
    case NUT_LENGTH_ERROR:
        throw std::length_error(message);
    case NUT_RANGE_ERROR:
        throw std::range_error(message);
    default:
        throw std::runtime_error(message);
    }
}

int current_device() {
    if (g_device < 0) {
        const char *env = std::getenv("NUTLLM_DEVICE");
        g_device = env != nullptr ? std::atoi(env) : 0;
    }
    return g_device;
}

void set_device(int device) { g_device = device; }

std::shared_ptr<nut_qmatrix> upload_qmatrix(const QuantizedMatrix &m) {
    nut_qmatrix_view view{};
    view.data = m.data().data();
    view.scales = m.scales().data();
    view.rows = int64_t(m.rows());
    view.cols = int64_t(m.cols());
    view.block_size = int64_t(m.block_size());
    view.type = m.type() == QuantType::int8 ? NUT_QUANT_INT8 : NUT_QUANT_INT4;
    nut_qmatrix *handle = nullptr;
    check(nut_qmatrix_create(&view, current_device(), &handle));
    return std::shared_ptr<nut_qmatrix>(handle, [](nut_qmatrix *h) {
        nut_qmatrix_destroy(h);
    });
}

} // namespace nutdev
