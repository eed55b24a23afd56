// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled via the runtime's
// driver entry point, so the library has no link dependency on libcuda).
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "tcgen05.cuh"

namespace b2 {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

int encode_tensor_map_3d_f16(CUtensorMap* map, const void* base, uint64_t inner_elems, uint64_t rows,
                             uint64_t batches, uint64_t row_stride_bytes, uint64_t batch_stride_bytes,
                             uint32_t box_inner, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return -1;
    if (batches <= 1) {
        batches = 1;
        batch_stride_bytes = (row_stride_bytes * rows + 15) / 16 * 16;
    }
    const cuuint64_t dims[3] = {inner_elems, rows, batches};
    const cuuint64_t strides[2] = {row_stride_bytes, batch_stride_bytes};
    const cuuint32_t box[3] = {box_inner, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -static_cast<int>(r);
}

int encode_token_rows_by_column_block(CUtensorMap* map, const void* base, uint64_t rows, uint32_t row_bytes,
                                      uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return -1;
    if (row_bytes % 128 != 0 || rows == 0) return -1;
    const cuuint64_t dims[3] = {64, rows, row_bytes / 128};
    const cuuint64_t strides[2] = {row_bytes, 128};
    const cuuint32_t box[3] = {64, box_rows, row_bytes / 128};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -static_cast<int>(r);
}

int encode_token_rows_by_column_block_seqs(CUtensorMap* map, const void* base, uint64_t rows, uint32_t row_bytes,
                                           uint64_t seqs, uint64_t seq_stride_bytes, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return -1;
    if (row_bytes % 128 != 0 || rows == 0 || seqs == 0 || seq_stride_bytes % 16 != 0) return -1;
    const cuuint64_t dims[4] = {64, rows, row_bytes / 128, seqs};
    const cuuint64_t strides[3] = {row_bytes, 128, seqs > 1 ? seq_stride_bytes : static_cast<uint64_t>(rows) * row_bytes};
    const cuuint32_t box[4] = {64, box_rows, row_bytes / 128, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -static_cast<int>(r);
}

}  // namespace b2
