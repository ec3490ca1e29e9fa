// q4_i8.cuh — launchers of the integer-MMA Q4 decode kernels (the default decode path).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q4_gemv.cuh"

namespace marlin {

// Activation rows per launch of the integer-MMA kernels (4 planes x 16 rows = 64 MMA columns).
constexpr int kI8MaxRows = 16;

// True when the integer-MMA kernels handle this shape: k a multiple of 512, at most 16384, and
// 1 <= m <= kI8MaxRows.
bool i8_supported(int64_t k, int64_t m);
// Decode GEMV family (same contract as launch_q4_gemv).
cudaError_t launch_i8_gemv(const GemvLaunch& L, cudaStream_t stream);
// Fused lm_head + argmax (same contract as launch_q4_lm_head_argmax).
cudaError_t launch_i8_lm_head(const LmHeadLaunch& L, cudaStream_t stream);
// Device error word of this translation unit (see gemv_device_error).
int i8_device_error(bool clear);
// Whole-row GEMV for one or two activation rows (q4_rows.cu): plain products (store epilogue, no
// RMSNorm, no planes in or out), k a multiple of 1024.  launch_i8_gemv takes it when it applies.
bool rows_gemv_applies(const GemvLaunch& L);
cudaError_t launch_rows_gemv(const GemvLaunch& L, cudaStream_t stream);
int rows_device_error(bool clear);

// Activation columns of the integer-MMA kernels for m rows (4 planes per row, MMA tiles of 8).
int i8_ncols(int64_t m);
// Bytes of the q, xs and xe arrays of an XPlanes set for m rows of k features (256-byte aligned
// pieces, q first), and the set laid out from `base` with the given ssq array.
size_t i8_planes_bytes(int64_t m, int64_t k);
XPlanes i8_planes_at(void* base, int64_t m, int64_t k, float* ssq, int nssq);

}  // namespace marlin
