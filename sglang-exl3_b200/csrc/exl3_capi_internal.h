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
}  // namespace exl3b200
