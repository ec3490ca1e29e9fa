// q4_misc.cuh — launchers for quantize/pack, RMSNorm, the Q4 embedding gather and the synthetic-input
// generator.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

namespace marlin {

enum : int { kDtypeBF16 = 0, kDtypeF32 = 1 };

cudaError_t launch_quantize(const uint16_t* w, int64_t n, int64_t k, uint32_t* wq, uint16_t* scales,
                            uint16_t* biases, cudaStream_t stream);
cudaError_t launch_rms_norm(const void* x, int dtype, const uint16_t* w, int64_t m, int64_t h, float eps,
                            float* out, cudaStream_t stream);
cudaError_t launch_residual_add(const void* h, int dtype, const float* y, int64_t n, float* out,
                                cudaStream_t stream);
cudaError_t launch_cast_bf16(const float* x, int64_t n, uint16_t* out, cudaStream_t stream);
cudaError_t launch_embed_q4(const int32_t* ids, int64_t m, const uint32_t* wq, const uint16_t* scales,
                            const uint16_t* biases, int64_t n, int64_t k, uint16_t* out, cudaStream_t stream);
int misc_device_error(bool clear);
cudaError_t launch_synth_bf16(uint16_t* out, int64_t n, uint64_t seed, float mean, float sigma, cudaStream_t stream);

}  // namespace marlin
