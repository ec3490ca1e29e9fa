// q4_host.cuh — host-side helpers shared by the TMA-fed Q4 kernels: tensor-map encoding of the MLX
// Q4 layout, the SM count and an extended launch (PDL / cluster attributes).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"
#include "q4_gemv.cuh"

namespace marlin {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (the library loads without a GPU).
inline EncodeTiledFn tmap_encode_fn() {
    // looked up once; the initialisation of a function-local static is thread-safe
    static const EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return EncodeTiledFn(nullptr);
    }();
    return fn;
}

// Tensor maps over one Q4 matrix: packed words as u32 [n][k/8] with box [32 words x box_rows] and
// 128-byte swizzle (one 128-byte line = 4 groups of a row); scales and biases as u16 [n][k/64]
// with box [8 groups x box_rows].  Rows past n read as zero.
inline bool encode_q4_maps(const Q4Mat& W, int box_rows, CUtensorMap* tw, CUtensorMap* ts, CUtensorMap* tb) {
    EncodeTiledFn fn = tmap_encode_fn();
    if (!fn) return false;
    const cuuint32_t es[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(W.k / 8), (cuuint64_t)W.n};
        const cuuint64_t strides[1] = {(cuuint64_t)(W.k / 2)};
        const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
        if (fn(tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(W.w), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)(W.k / 64), (cuuint64_t)W.n};
    const cuuint64_t strides[1] = {(cuuint64_t)(W.k / 64 * 2)};
    const cuuint32_t box[2] = {8, (cuuint32_t)box_rows};
    for (int i = 0; i < 2; ++i) {
        if (fn(i ? tb : ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(i ? W.b : W.s), dims, strides, box,
               es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

inline int device_num_sms() { return device_sm_count(); }

// cudaLaunchKernelEx with optional programmatic stream serialization and cluster dimension.
template <typename KernelT, typename ArgT>
cudaError_t launch_ex(KernelT kernel, const ArgT& args, int grid, int threads, int cluster, uint32_t smem, bool pdl,
                      cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

// Host read (and optional clear) of this translation unit's device error word.
inline int tu_device_error(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_marlin_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_marlin_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

}  // namespace
}  // namespace marlin
