#pragma once
/* Glue between the C++ host API and the C ABI of libnutcuda.so: status
 * codes become the exception classes the reference throws for the same
 * condition, and device handles are owned by shared pointers. */
#include <memory>

#include "../../include/nutllm_cuda.h"

class QuantizedMatrix;

namespace nutdev {

/* Throws std::invalid_argument / out_of_range / length_error / range_error
 * / runtime_error for the matching nut_status, with nut_last_error(). */
void check(nut_status status);

/* Device the host API places new device objects on (default 0, or the
 * NUTLLM_DEVICE environment variable). */
int current_device();
void set_device(int device);

std::shared_ptr<nut_qmatrix> upload_qmatrix(const QuantizedMatrix &matrix);

} // namespace nutdev
