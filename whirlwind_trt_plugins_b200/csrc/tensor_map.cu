// tensor_map.cu -- see tensor_map.cuh.
#include "tensor_map.cuh"

#include <mutex>

namespace ww {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() noexcept
{
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            cudaGetLastError();  // leave no sticky error behind
    });
    return fn;
}

}  // namespace

bool encode_feature_map(CUtensorMap* out, const void* base, int B, int C, int rows, int W, int box_x, int box_z,
                        bool swizzle128) noexcept
{
    if (out == nullptr || base == nullptr || B <= 0 || C <= 0 || rows <= 0 || W <= 0) return false;
    if (W % 8 != 0 || reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
    if (box_x <= 0 || box_x > 256 || box_z <= 0 || box_z > 256 || (box_x * 2) % 16 != 0) return false;
    if (swizzle128 && box_x * 2 > 128) return false;
    const EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(rows),
                                static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(B)};
    const cuuint64_t row_b = static_cast<cuuint64_t>(W) * 2;
    const cuuint64_t strides[3] = {row_b, row_b * rows, row_b * rows * C};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(box_x), 1u, static_cast<cuuint32_t>(box_z), 1u};
    const cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
    const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool encode_volume_map(CUtensorMap* out, const void* base, int B, int G, int D, int H, int W, int box_x, int box_d,
                       int box_g) noexcept
{
    if (out == nullptr || base == nullptr || B <= 0 || G <= 0 || D <= 0 || H <= 0 || W <= 0) return false;
    if (W % 8 != 0 || reinterpret_cast<uintptr_t>(base) % 16 != 0) return false;
    if (box_x <= 0 || box_x > 256 || (box_x * 2) % 16 != 0) return false;
    if (box_d <= 0 || box_d > 256 || box_g <= 0 || box_g > 256) return false;
    const EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    const cuuint64_t dims[5] = {static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(D),
                                static_cast<cuuint64_t>(G), static_cast<cuuint64_t>(B)};
    const cuuint64_t row_b = static_cast<cuuint64_t>(W) * 2;
    const cuuint64_t plane_b = row_b * static_cast<cuuint64_t>(H);
    const cuuint64_t strides[4] = {row_b, plane_b, plane_b * D, plane_b * D * G};
    const cuuint32_t box[5] = {static_cast<cuuint32_t>(box_x), 1u, static_cast<cuuint32_t>(box_d),
                               static_cast<cuuint32_t>(box_g), 1u};
    const cuuint32_t estr[5] = {1u, 1u, 1u, 1u, 1u};
    const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace ww
