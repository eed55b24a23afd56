// CUDA equivalents of the reference's include/gpu_utils.hpp helpers that the
// attention path needs: a checking macro and last_captured_node.
#pragma once

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "b200attn.h"

// include/gpu_utils.hpp:7-14 HIP_CHECK: print and exit on a runtime error.
#define B2_CUDA_CHECK(command)                                                              \
    do {                                                                                    \
        cudaError_t b2_status_ = (command);                                                 \
        if (b2_status_ != cudaSuccess) {                                                    \
            std::fprintf(stderr, "[CUDA Error] %s at %s:%d\n", cudaGetErrorString(b2_status_), \
                         __FILE__, __LINE__);                                               \
            std::exit(EXIT_FAILURE);                                                        \
        }                                                                                   \
    } while (0)

namespace b200attn {

// Throw for a negative b2 status (the C ABI never throws itself).
inline int check(int status, const char* where) {
    if (status < 0)
        throw std::runtime_error(std::string(where) + ": " + b2_status_string(status));
    return status;
}

// include/gpu_utils.hpp:45-58 last_captured_node.
inline cudaGraphNode_t last_captured_node(cudaStream_t stream) {
    cudaStreamCaptureStatus capture_status;
    const cudaGraphNode_t* dependencies = nullptr;
    size_t count = 0;
    B2_CUDA_CHECK(cudaStreamGetCaptureInfo(stream, &capture_status, nullptr, nullptr, &dependencies, &count));
    if (capture_status != cudaStreamCaptureStatusActive || count != 1)
        throw std::runtime_error("Expected one capture dependency");
    return dependencies[0];
}

}  // namespace b200attn
