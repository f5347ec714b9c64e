// tma_host.h -- host-side TMA tensor-map creation (driver entry point fetched
// through the runtime, so the library needs no link-time libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace gdn {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (fn == nullptr) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Tensor map over a bf16 [T][H][128] tensor (token-major, head, head dim) whose
// box is 64 head-dim elements x 1 head x 64 tokens, written to shared memory
// with the 128-byte swizzle: one box = one K-major SW128 atom column of 64
// token rows.  Out-of-range tokens read as zero.
inline bool make_tmap_thd_bf16(CUtensorMap *map, const void *base, int64_t T, int H) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr || T <= 0 || H <= 0) return false;
    cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(T)};
    cuuint64_t strides[2] = {128 * 2, static_cast<cuuint64_t>(H) * 128 * 2};
    cuuint32_t box[3] = {64, 1, 64};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace gdn
