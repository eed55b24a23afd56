// HIP -> CUDA type aliases, so engine code written against the reference's
// include/kernels/kernels.hpp compiles unchanged on the CUDA build.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#ifndef __HIP_PLATFORM_AMD__
using hipStream_t = cudaStream_t;
using hipGraph_t = cudaGraph_t;
using hipGraphExec_t = cudaGraphExec_t;
using hipGraphNode_t = cudaGraphNode_t;
using hipError_t = cudaError_t;
#endif
