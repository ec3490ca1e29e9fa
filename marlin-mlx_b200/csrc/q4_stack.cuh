// q4_stack.cuh — launcher of the one-kernel Q4 layer stack of the decode step (persistent, cooperative).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "q4_gemv.cuh"

namespace marlin {

constexpr int kStackMaxLayers = 24;  // tensor maps travel as kernel parameters (<= 32 KB)
constexpr int kStackMaxRows = 4;  // activation planes share shared memory with the ring

struct StackLayer {
    const uint16_t* norm;  // post-attention RMSNorm weight (1 + w), bf16 [hidden]
    Q4Mat gate, up, down;
};

struct StackLaunch {
    const void* h0;  // [m, hidden] input rows (bf16 or binary32)
    int h0_dtype;
    int64_t m, hidden, inter;
    int n_layers;
    const StackLayer* layers;
    float eps;
    float* h_out;     // optional [m, hidden] binary32 for the last layer's output (else in scratch)
    unsigned* bar;    // control block of 64 words, zero before the first launch (left zero)
    void* scratch;    // >= stack_scratch_size bytes, 256-byte aligned (no initial contents needed)
};

bool stack_supported(int64_t m, int64_t hidden, int64_t inter, int n_layers);
size_t stack_scratch_size(int64_t m, int64_t hidden, int64_t inter);
cudaError_t launch_stack(const StackLaunch& L, cudaStream_t stream);
// Where the last layer's output lands: h_out, or inside the scratch.
inline float* stack_output(const StackLaunch& L) {
    return L.h_out ? L.h_out : reinterpret_cast<float*>(L.scratch) + 2 * L.m * L.hidden;
}
int stack_device_error(bool clear);

}  // namespace marlin
