// q4_prefill.cuh — launcher of the tcgen05 Q4 GEMM for prefill-sized activations.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q4_gemv.cuh"

namespace marlin {

// Activation rows above which bf16 inputs go to the tcgen05 GEMM instead of the decode kernels.
constexpr int64_t kPrefillMinRows = 16;

// True when the GEMM handles this launch: bf16 activations without a fused RMSNorm, m above
// kPrefillMinRows, k a multiple of 512.
bool prefill_applies(const GemvLaunch& L);
// All m rows in one persistent launch (same contract as launch_q4_gemv).
cudaError_t launch_prefill(const GemvLaunch& L, cudaStream_t stream);
// Device error word of this translation unit (see gemv_device_error).
int prefill_device_error(bool clear);

}  // namespace marlin
