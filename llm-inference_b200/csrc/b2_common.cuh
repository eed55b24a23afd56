// Shared helpers of the b200attn CUDA library (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "b200attn.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "b200attn is built for sm_100a only"
#endif

namespace b2 {

// Library-wide bookkeeping (b2_status.cu).
void note_cuda_error(cudaError_t e);
void count_launch(uint64_t n = 1);
// Device error words of the translation units with bounded waits.
unsigned int device_error_decode();
unsigned int device_error_prefill();
int clear_device_error_decode();
int clear_device_error_prefill();
unsigned int device_error_ragged();
int clear_device_error_ragged();
unsigned int device_error_proj();
int clear_device_error_proj();

// Turn the launch status of the kernel just enqueued into a b2 status.
inline int launch_status() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    count_launch();
    return B2_OK;
}

inline int cuda_status(cudaError_t e) {
    if (e != cudaSuccess) {
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    return B2_OK;
}

// Launch with programmatic dependent launch allowed: the kernel may start
// while the previous kernel on the stream finishes; every kernel launched this
// way executes griddepcontrol.wait before reading memory a predecessor writes.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        note_cuda_error(e);
        return B2_ERR_CUDA;
    }
    return launch_status();
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The node most recently added to a capturing stream (the CUDA form of the
// reference's last_captured_node, include/gpu_utils.hpp:45-58).
int last_captured_node(cudaStream_t stream, cudaGraphNode_t* node);

// Read a captured kernel node's parameters, check that it runs `expected`
// (one of this library's kernels) and return its parameter block.
int node_kernel_params(cudaGraphNode_t node, const void* const* expected, int n_expected,
                       cudaKernelNodeParams* params);

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Rotate-half RoPE of 8 pairs: lo holds x[i..i+8) of a head, hi holds
// x[i+d/2..i+d/2+8), cv/sv the fp16 cos/sin of frequencies i..i+8. fp32
// x0*c - x1*s and x1*c + x0*s with every product and sum rounded separately
// (no FMA contraction), then round-to-nearest fp16: the reference's
// arithmetic (src/kernels/rope.hip.cpp:61-134), bit-identical to the CPU
// oracle evaluated the same way.
__device__ __forceinline__ void rot8_pairs(uint4& lo, uint4& hi, uint4 cv, uint4 sv) {
    uint32_t* L = reinterpret_cast<uint32_t*>(&lo);
    uint32_t* Hh = reinterpret_cast<uint32_t*>(&hi);
    const uint32_t* C = reinterpret_cast<const uint32_t*>(&cv);
    const uint32_t* S = reinterpret_cast<const uint32_t*>(&sv);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const float2 x0 = __half22float2(*reinterpret_cast<const __half2*>(&L[w]));
        const float2 x1 = __half22float2(*reinterpret_cast<const __half2*>(&Hh[w]));
        const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&C[w]));
        const float2 sn = __half22float2(*reinterpret_cast<const __half2*>(&S[w]));
        const float a0 = __fsub_rn(__fmul_rn(x0.x, c.x), __fmul_rn(x1.x, sn.x));
        const float a1 = __fsub_rn(__fmul_rn(x0.y, c.y), __fmul_rn(x1.y, sn.y));
        const float b0 = __fadd_rn(__fmul_rn(x1.x, c.x), __fmul_rn(x0.x, sn.x));
        const float b1 = __fadd_rn(__fmul_rn(x1.y, c.y), __fmul_rn(x0.y, sn.y));
        L[w] = pack_half2(a0, a1);
        Hh[w] = pack_half2(b0, b1);
    }
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

}  // namespace b2
