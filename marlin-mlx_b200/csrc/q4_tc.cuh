// q4_tc.cuh — launchers of the tcgen05 (TMEM) decode kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q4_gemv.cuh"

namespace marlin {

// True when the tcgen05 kernels handle this shape: k a multiple of 512 and m * planes <= 32.
bool tc_supported(int64_t k, int64_t m_eff);
// Whether the tcgen05 kernel's shared-memory plan fits for this launch (else use mma.sync).
bool tc_gemv_fits(const GemvLaunch& L);
bool tc_lm_head_fits(const LmHeadLaunch& L);
// Decode GEMV family on tcgen05 (same contract as launch_q4_gemv).
cudaError_t launch_tc_gemv(const GemvLaunch& L, cudaStream_t stream);
// Fused lm_head + argmax on tcgen05 (same contract as launch_q4_lm_head_argmax).
cudaError_t launch_tc_lm_head(const LmHeadLaunch& L, cudaStream_t stream);
// Device error word of this translation unit (see gemv_device_error).
int tc_device_error(bool clear);

}  // namespace marlin
