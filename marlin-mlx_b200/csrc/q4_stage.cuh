// q4_stage.cuh — activation loading and RMSNorm factors shared by the Q4 decode kernels.
#pragma once

#include "common.cuh"
#include "q4_gemv.cuh"

namespace marlin {
namespace {

constexpr int kGroup = 64;

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// ------------------------------------------------------------------------------------------------
// activation staging
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float load_act(const void* x, int dtype, int64_t i) {
    if (dtype == kBF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(x)[i]);
    return static_cast<const float*>(x)[i];
}

struct XGeom {
    uint8_t* xp;  // planes: row r = plane*M + m, stride XRS bytes, GC groups of 128 B
    float* xs;    // [M_eff][GC] plane sums per group
    float* rf;    // [M] RMSNorm factors
    float* ssq;   // [M * K/8] per-unit sums of squares (norm only)
    int M, P, M_eff, XRS, GC;
};

// Counted fixed point, the one-kernel layer stack's accumulator of h: a 64-bit two's-complement
// word holds (value * 2^27) << 5 plus, in its low 5 bits, the number of contributions added so far
// (each atomic add carries +1 there), so a reader knows from the word itself when it is complete.
constexpr int kFixCountBits = 5;
constexpr float kFixUnit = 7.450580596923828125e-9f;  // 2^-27

__device__ __forceinline__ float fix_value(unsigned long long w) {
    return __ll2float_rn((long long)w >> kFixCountBits) * kFixUnit;
}

// Eight consecutive counted fixed-point words (complete ones) as binary32, read from L2.
__device__ __forceinline__ void load_fix8(const unsigned long long* p, float v[8]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const ulonglong2 q = __ldcg(reinterpret_cast<const ulonglong2*>(p) + k);
        v[2 * k] = fix_value(q.x);
        v[2 * k + 1] = fix_value(q.y);
    }
}

// Eight consecutive activations starting at element i (i % 8 == 0), as binary32.
__device__ __forceinline__ void load8(const void* x, int dtype, int64_t i, float v[8]) {
    if (dtype == kFix64) {
        load_fix8(static_cast<const unsigned long long*>(x) + i, v);
    } else if (dtype == kBF16) {
        const uint4 r = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + i);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] = bf16_bits_to_f32(w[j] & 0xffffu);
            v[2 * j + 1] = bf16_bits_to_f32(w[j] >> 16);
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + i);
        const float4 b = *reinterpret_cast<const float4*>(static_cast<const float*>(x) + i + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

// Sum of squares of one 8-element unit as MLX's C++ rms_norm evaluates mean(square(x))
// (src/model/marlin.cpp:13): bf16 x squares round to bf16; binary32 x stays binary32.
__device__ __forceinline__ float unit_ssq(const float v[8], int dtype) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float sq = __fmul_rn(v[j], v[j]);
        if (dtype == kBF16) sq = bf16_round(sq);
        s = __fadd_rn(s, sq);
    }
    return s;
}

// Row factors r_m = 1/sqrt(mean + eps) from the per-unit sums in g.ssq (fixed order: units
// lane-strided, then a shuffle tree).  bf16 x: the sum and the mean round to bf16; the `+ eps`
// (a C++ float, src/core/config.h:20) and everything after it is binary32.  Ends with a barrier.
__device__ void finish_norm_factors(int dtype, int M, int K, float eps, const XGeom& g) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int upr = K / 8;
    for (int m = warp; m < M; m += nw) {
        float s = 0.f;
        for (int u = lane; u < upr; u += 32) s = __fadd_rn(s, g.ssq[m * upr + u]);
#pragma unroll
        for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) {
            float var;
            if (dtype == kBF16)
                var = bf16_round(__fmul_rn(bf16_round(s), bf16_round((float)(1.0 / (double)K))));
            else
                var = __fmul_rn(s, (float)(1.0 / (double)K));
            g.rf[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
        }
    }
    __syncthreads();
}

__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo, uint32_t hi) { return lo | (hi << 16); }

// Emit one 8-element unit (row m, unit ul of the staged chunk): optional RMSNorm, split into
// planes, one 16-byte store per plane at slot positions 8*(ul & 1) + {0,2,4,6,1,3,5,7}, and the
// plane sums of the unit's 64-group (the 8 units of a group are 8 consecutive lanes: a 3-step
// shuffle tree).  Every lane of the warp must call it (ok = false contributes nothing).
__device__ __forceinline__ void emit_unit(float (&v)[8], uint4 nwv, int m, int ul, bool ok, bool normed,
                                          const XGeom& g) {
    const int lane = threadIdx.x & 31, P = g.P;
    float ps[3] = {0.f, 0.f, 0.f};
    if (ok) {
        if (normed) {
            const float r = g.rf[m];
            const uint32_t w4[4] = {nwv.x, nwv.y, nwv.z, nwv.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float wj = bf16_bits_to_f32((w4[j >> 1] >> (16 * (j & 1))) & 0xffffu);
                v[j] = __fmul_rn(__fmul_rn(v[j], r), __fadd_rn(1.0f, wj));
            }
        }
        uint32_t h[3][8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            h[0][j] = f32_to_bf16_bits(v[j]);
            if (P == 3) {
                const float r1 = __fsub_rn(v[j], bf16_bits_to_f32(h[0][j]));
                h[1][j] = f32_to_bf16_bits(r1);
                h[2][j] = f32_to_bf16_bits(__fsub_rn(r1, bf16_bits_to_f32(h[1][j])));
            }
        }
        const int gl = ul >> 3, e0 = (ul & 7) * 8;
        const uint32_t off = gl * 128 + (e0 >> 4) * 32 + ((e0 >> 3) & 1) * 16;
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            if (p < P) {
                uint4 st;
                st.x = pack_bf16x2(h[p][0], h[p][4]);
                st.y = pack_bf16x2(h[p][1], h[p][5]);
                st.z = pack_bf16x2(h[p][2], h[p][6]);
                st.w = pack_bf16x2(h[p][3], h[p][7]);
                *reinterpret_cast<uint4*>(g.xp + (uint32_t)(p * g.M + m) * g.XRS + off) = st;
                float s = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) s += bf16_bits_to_f32(h[p][j]);
                ps[p] = s;
            }
        }
    }
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        if (p < P) {
            float s = ps[p];
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            s += __shfl_xor_sync(0xffffffffu, s, 4);
            if (ok && (lane & 7) == 0) g.xs[(p * g.M + m) * g.GC + (ul >> 3)] = s;
        }
    }
}

// Stage activation groups [gc0, gc0 + ngc) of x[M, K] into g (RMSNorm factors must already be in
// g.rf when norm_w is set).  Loads of a pass are all issued before use.  Ends with __syncthreads.
__device__ void stage_chunk(const void* x, int dtype, int K, const uint16_t* norm_w, int gc0, int ngc,
                            const XGeom& g) {
    const int nt = blockDim.x, lane = threadIdx.x & 31;
    const int upr = ngc * 8, total = g.M * upr;
    const int k0c = gc0 * kGroup;
    constexpr int U = 2;
    for (int base = (int)threadIdx.x - lane; base < total; base += nt * U) {  // warp-uniform trip count
        float v[U][8];
        uint4 nwv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = base + lane + u * nt;
            if (idx < total) {
                const int m = idx / upr, k = k0c + (idx % upr) * 8;
                load8(x, dtype, (int64_t)m * K + k, v[u]);
                if (norm_w) nwv[u] = *reinterpret_cast<const uint4*>(norm_w + k);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = base + lane + u * nt;
            const bool ok = idx < total;
            emit_unit(v[u], nwv[u], ok ? idx / upr : 0, ok ? idx % upr : 0, ok, norm_w != nullptr, g);
        }
    }
    __syncthreads();
}

// Per-unit sums of squares of the whole x[M, K] into g.ssq, then the row factors.
__device__ void norm_factors_only(const void* x, int dtype, int K, float eps, const XGeom& g) {
    const int nt = blockDim.x, upr = K / 8, total = g.M * upr;
    for (int base = (int)threadIdx.x; base < total; base += nt * 2) {
        float v[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = base + u * nt;
            if (idx < total) load8(x, dtype, (int64_t)(idx / upr) * K + (idx % upr) * 8, v[u]);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = base + u * nt;
            if (idx < total) g.ssq[idx] = unit_ssq(v[u], dtype);
        }
    }
    __syncthreads();
    finish_norm_factors(dtype, g.M, K, eps, g);
}

}  // namespace
}  // namespace marlin
