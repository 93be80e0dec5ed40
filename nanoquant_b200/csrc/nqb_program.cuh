// Internal declarations of the persistent decode program of libnqb.
#pragma once

#include "nqb_common.cuh"

namespace nqb {

// Reads and clears the program kernel's device status word.
int program_device_error(int32_t *out);

}  // namespace nqb
