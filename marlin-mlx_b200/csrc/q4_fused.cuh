// q4_fused.cuh — launcher of the one-kernel MLP layer stack of the decode step (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q4_gemv.cuh"

namespace marlin {

// Layers per launch: every layer's nine tensor maps travel in the kernel parameters (32 KB limit).
constexpr int kFusedMaxLayers = 24;
// Activation rows per launch (four planes each: 32 MMA columns).
constexpr int kFusedMaxRows = 8;

struct FusedLayer {
    const uint16_t* norm_w;  // bf16 [hidden] RMSNorm weight (multiplier 1 + w)
    Q4Mat gate, up, down;
};

// The Q4 sublayers of n_layers decoder layers on m activation rows:
//   h <- h + down(swiglu(gate(rms_norm(h)), up(rms_norm(h))))
// h starts as the bf16 rows h0 [m][hidden]; the result stays in acc (see below) for the lm_head.
struct FusedLaunch {
    const uint16_t* h0;
    int64_t m, hidden, inter;
    int n_layers;
    const FusedLayer* layers;
    float eps;
    // Three [m][hidden] 64-bit counted fixed-point accumulators (two's complement: (value * 2^27)
    // << 5 plus a 5-bit count of the contributions added); after the launch the final h is
    // acc[n_layers % 3].  No state is carried between launches in them.
    unsigned long long* acc;
    // Two words: the arrival counter of the layer barriers and the abort word.  Zero on entry; left
    // non-zero, the next kernel in the stream must clear them (the lm_head kernel does, see
    // LmHeadLaunch::reset) before another launch.
    unsigned* sync;
    unsigned long long wait_cycles;  // bound of each wait (SM clock cycles)
    bool pdl;
};

// Shapes the kernel serves: m <= kFusedMaxRows, hidden in {512, 1024, 2048}, inter a multiple of
// 512 with inter / 64 CTAs co-resident on this device (one per SM, clusters of 8),
// n_layers <= kFusedMaxLayers, and every layer with the same shapes.
bool fused_supported(int64_t m, int64_t hidden, int64_t inter, int n_layers);
size_t fused_acc_bytes(int64_t m, int64_t hidden);
cudaError_t launch_fused_layers(const FusedLaunch& F, cudaStream_t stream);
int fused_device_error(bool clear);

}  // namespace marlin
