// Internal include for the C-ABI translation units: the public header plus the
// standard headers the host-side launch code needs.
#pragma once

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "exl3_b200.h"

namespace exl3b200 {
// device address of the library's sticky device status (exl3_tc.cu); null on error
int* exl3_status_dev_ptr();
// limit of a bounded device-side wait for kernels launched now: the value set by
// exl3b200_set_wait_limit, or dflt when none is set
unsigned long long wait_limit_ns(unsigned long long dflt);
}  // namespace exl3b200
