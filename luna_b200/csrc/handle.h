// handle.h -- the opaque lb200_model handle of the C ABI.
#pragma once

#include "engine.h"

#include <string>

namespace lb200 {
// Record msg as this thread's lb200_last_error() text; returns 1.
int set_last_error(const std::string& msg);
}  // namespace lb200

struct lb200_model {
    lb200::Model* m = nullptr;
    cudaStream_t stream = nullptr;
};
