// q4_i8_common.cuh — pieces of the integer-MMA Q4 decode path shared by its kernels: activation
// staging into four exact s8 planes (with the fused RMSNorm) and the per-stage tensor-core step.
// Staging is written for a "team" of threads (the whole block, or the consumer warps of a
// warp-specialised kernel) that synchronises through team.sync().
#pragma once

#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_stage.cuh"

// Optional timeline hook inside the activation staging (point 0..3), empty in the library build.
#ifndef STAGE_MARK
#define STAGE_MARK(k)
#endif

namespace marlin {
namespace {

constexpr uint32_t kNib = 0x0F0F0F0Fu;

// Every thread of the block.
struct BlockTeam {
    __device__ __forceinline__ int size() const { return blockDim.x; }
    __device__ __forceinline__ int rank() const { return threadIdx.x; }
    __device__ __forceinline__ void sync() { __syncthreads(); }
};

// RMSNorm factors r_m = 1/sqrt(mean + eps) from the per-unit sums t.ssq, in the fixed order of
// finish_norm_factors (units lane-strided, then a shuffle tree).  Ends with team.sync().
template <class Team>
__device__ void norm_factors_team(Team& team, int dtype, int M, int K, float eps, float* rf, const float* ssq) {
    const int lane = team.rank() & 31, warp = team.rank() >> 5, nw = team.size() >> 5;
    const int upr = K / 8;
    for (int m = warp; m < M; m += nw) {
        float s = 0.f;
        for (int u = lane; u < upr; u += 32) s = __fadd_rn(s, ssq[m * upr + u]);
#pragma unroll
        for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) {
            float var;
            if (dtype == kBF16)
                var = bf16_round(__fmul_rn(bf16_round(s), bf16_round((float)(1.0 / (double)K))));
            else
                var = __fmul_rn(s, (float)(1.0 / (double)K));
            rf[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
        }
    }
    team.sync();
}

// ------------------------------------------------------------------------------------------------
// activation staging: four s8 planes per row, [group][column][64 B] with column = 4 m + p.
// Within a group's 64 bytes, unit u (elements 8u..8u+7) occupies bytes 8u..8u+7 as
// (x0, x2, x4, x6, x1, x3, x5, x7): the order the B fragment of mma.m16n8k32 needs when the A
// fragment is (q0, q2, q4, q6 | q1, q3, q5, q7) of one packed word.
// ------------------------------------------------------------------------------------------------
//
// Fold.  With e the exponent of a group's planes (|x| < 2^e), x = 2^(e-6) sum_p 128^-p i_p, so per
// weight row and 64-group, s * sum(q x) + b * sum(x) = 2^-6 sum_p 128^-p (s 2^e D_p) + b sum(x).
// The codes enter two MMAs without shifting: the even elements as q (w & 0x0F0F0F0F) and the odd
// ones as 16 q (w & 0xF0F0F0F0, unsigned bytes), so 16 D_p = 16 D_even + D_odd' exactly.  The
// kernels accumulate Y_p += (s * xe) * 16 D_p and, per row, Yb += b * xs (xs = 64 sum(x), held on
// the plane-0 columns), and combine once per output: sum_p cs_p Y_p + 2^-6 Yb with
// cs = 2^(-10-7p).  Every scaling is by a power of two, so the exponent may vary per group (planes
// written by the producing kernel) or be one per row (planes staged here) with the same arithmetic.
struct I8X {
    uint8_t* xq;          // [ng][ncols][64]
    float* xs;            // [ng][ncols]: plane-0 columns hold 64 sum_g(x), the others 0
    float* cs;            // [ncols]: 2^(-6-7p) (0 for padding columns)
    float* rf;            // [M] RMSNorm factors
    float* ssq;           // [M * K/8] RMSNorm scratch
    unsigned int* amax;   // [M] max |x| (binary32 bits) over the staged range
    float* xe;            // [ng][ncols]: 2^e of the group's planes (0 for padding columns)
};

// One 64-group of a warp's 16-row weight tile against activation column tile j (see Fold): wa, wb
// the lane's packed words 2t, 2t + 1 of rows g and g + 8; xv the lane's 16 plane bytes (elements
// 16t..16t+15 of column g, evens then odds per 8); sr/br the rows' scales and biases; xe and x0
// the group's 2^e and 64 sum(x) for the lane's activation row.  y: rows g, g+8 x columns 2t, 2t+1.
__device__ __forceinline__ void i8_group(uint2 wa, uint2 wb, uint4 xv, float sr0, float sr1, float br0, float br1,
                                         float xe, float x0, float (&y)[4], float (&yb)[2]) {
    const uint32_t lo[4] = {wa.x & kNib, wb.x & kNib, wa.y & kNib, wb.y & kNib};
    const uint32_t hi[4] = {wa.x & ~kNib, wb.x & ~kNib, wa.y & ~kNib, wb.y & ~kNib};
    int c[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0};
    mma_u8s8_16832(c, lo, xv.x, xv.z);  // even elements
    mma_u8s8_16832(e, hi, xv.y, xv.w);  // odd elements, times 16
    const float s0 = sr0 * xe, s1 = sr1 * xe;
    y[0] = fmaf(s0, (float)(16 * c[0] + e[0]), y[0]);
    y[1] = fmaf(s0, (float)(16 * c[1] + e[1]), y[1]);
    y[2] = fmaf(s1, (float)(16 * c[2] + e[2]), y[2]);
    y[3] = fmaf(s1, (float)(16 * c[3] + e[3]), y[3]);
    yb[0] = fmaf(br0, x0, yb[0]);
    yb[1] = fmaf(br1, x0, yb[1]);
}

// i8_group for wide column tiles: the even codes enter as 16 q ((w << 4) & 0xF0F0F0F0) so both MMAs
// chain into one accumulator that starts at the bits of 1.5 * 2^23; read back as binary32 minus
// 1.5 * 2^23 it is exactly 16 D_even + D_odd' (|.| < 2^20), so the fold needs no int-to-float
// conversion and runs as packed pairs.  Same bits as i8_group.
__device__ __forceinline__ void i8_group_chained(uint2 wa, uint2 wb, uint4 xv, float sr0, float sr1, float br0,
                                                 float br1, float xe, float x0, float (&y)[4], float (&yb)[2]) {
    const uint32_t lo[4] = {(wa.x << 4) & ~kNib, (wb.x << 4) & ~kNib, (wa.y << 4) & ~kNib, (wb.y << 4) & ~kNib};
    const uint32_t hi[4] = {wa.x & ~kNib, wb.x & ~kNib, wa.y & ~kNib, wb.y & ~kNib};
    int d[4] = {0x4B400000, 0x4B400000, 0x4B400000, 0x4B400000};
    mma_u8s8_16832(d, lo, xv.x, xv.z);  // even elements, times 16
    mma_u8s8_16832(d, hi, xv.y, xv.w);  // odd elements, times 16
    fold_pair(y[0], y[1], (uint32_t)d[0], (uint32_t)d[1], sr0 * xe);
    fold_pair(y[2], y[3], (uint32_t)d[2], (uint32_t)d[3], sr1 * xe);
    yb[0] = fmaf(br0, x0, yb[0]);
    yb[1] = fmaf(br1, x0, yb[1]);
}

// The outputs of a lane after the K loop: rows g (.x) and g + 8 (.y) of activation row
// m = 2j + (t >> 1), summed over the lane pair (t, t ^ 1) that holds the row's four planes.
__device__ __forceinline__ float2 i8_combine(const float (&y)[4], const float (&yb)[2], float2 cv, int tq) {
    const float bw = (tq & 1) ? 0.f : 0.015625f;  // 2^-6 Yb, added once per pair
    float p0 = fmaf(bw, yb[0], fmaf(cv.x, y[0], cv.y * y[1]));
    float p1 = fmaf(bw, yb[1], fmaf(cv.x, y[2], cv.y * y[3]));
    p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
    p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
    return make_float2(p0, p1);
}

// byte offset of element k (0..63) of a group in its 64-byte plane row (B-fragment order)
__device__ __forceinline__ int plane_pos(int k) {
    const int j = k & 7;
    return (k & ~7) + ((j & 1) ? 4 : 0) + (j >> 1);
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// exponent e with max|x| < 2^e (clamped so that every plane scale stays a normal binary32)
__device__ __forceinline__ int row_exp(unsigned int abits) {
    const int eb = (int)((abits >> 23) & 0xffu);
    const int e = eb == 0 ? -125 : eb - 126;
    return max(e, -90);
}

// Eight activations of row m from column k, RMSNorm'ed as marlin.cpp:12-16 when norm_w is set.
__device__ __forceinline__ void load_norm8(const void* x, int dtype, int K, const uint16_t* norm_w, const float* rf,
                                           int m, int k, float (&v)[8]) {
    load8(x, dtype, (int64_t)m * K + k, v);
    if (norm_w) {
        const uint4 nwv = *reinterpret_cast<const uint4*>(norm_w + k);
        const uint32_t w4[4] = {nwv.x, nwv.y, nwv.z, nwv.w};
        const float r = rf[m];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float wj = bf16_bits_to_f32((w4[j >> 1] >> (16 * (j & 1))) & 0xffffu);
            v[j] = __fmul_rn(__fmul_rn(v[j], r), __fadd_rn(1.0f, wj));
        }
    }
}

// Max over the warp of `bits` for the lanes whose row is m0, and for row m1 when the warp's 32
// consecutive units straddle two rows; one shared-memory atomic per row and warp.
__device__ __forceinline__ void warp_row_max(unsigned int* amax, unsigned int bits, int m, int base, int total, int upr) {
    const int m0 = base / upr, m1 = min(base + 31, total - 1) / upr;
    const unsigned int r0 = __reduce_max_sync(0xffffffffu, m == m0 ? bits : 0u);
    if ((threadIdx.x & 31) == 0) atomicMax(&amax[m0], r0);
    if (m1 != m0) {
        const unsigned int r1 = __reduce_max_sync(0xffffffffu, m == m1 ? bits : 0u);
        if ((threadIdx.x & 31) == 0) atomicMax(&amax[m1], r1);
    }
}

// The four s8 planes of eight activations with row exponent e (|x| < 2^e, up to rounding):
// x = 2^(e-13) A + 2^(e-27) B with integers |A|, |B| <= 2^13 + 8 (both steps exact), then each of
// A, B splits into two balanced base-128 digits: A = 128 i0 + i1, i1 in [-64, 63].  Bytes go out in
// the B-fragment order (x0, x2, x4, x6 | x1, x3, x5, x7).
__device__ __forceinline__ void planes8(const float (&v)[8], int e, uint32_t (&b)[4][2]) {
    const float s1 = pow2f(13 - e), d1 = pow2f(e - 13), s2 = pow2f(27 - e);
#pragma unroll
    for (int p = 0; p < 4; ++p) b[p][0] = b[p][1] = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float qa = rintf(__fmul_rn(v[j], s1));
        const int A = (int)qa;
        const int B = __float2int_rn(__fmul_rn(fmaf(-qa, d1, v[j]), s2));
        const int i0 = (A + 64) >> 7, i2 = (B + 64) >> 7;
        const int d[4] = {i0, A - (i0 << 7), i2, B - (i2 << 7)};
#pragma unroll
        for (int p = 0; p < 4; ++p) b[p][j & 1] |= ((uint32_t)d[p] & 0xffu) << (8 * (j >> 1));
    }
}

// RMSNorm of eight activations as marlin.cpp:12-16: (x * r) * (1 + w), binary32.
__device__ __forceinline__ void norm8(float (&v)[8], uint4 nwv, float r) {
    const uint32_t w4[4] = {nwv.x, nwv.y, nwv.z, nwv.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float wj = bf16_bits_to_f32((w4[j >> 1] >> (16 * (j & 1))) & 0xffffu);
        v[j] = __fmul_rn(__fmul_rn(v[j], r), __fadd_rn(1.0f, wj));
    }
}

constexpr int kStageU = 2;  // 8-element activation units per thread and chunk, held in registers

// Stage groups [g0, g0 + ng) of the M activation rows (ng % 4 == 0).  All threads of the block
// call it; it ends with a barrier.  The rows are read in chunks of kStageU units per thread (whole
// rows when RMSNorm applies, since its factor needs every column; else only the staged range).
// With one chunk, x is read from global memory once and the norm sums, row maxima and planes come
// from registers; larger inputs read each chunk twice.
template <class Team>
__device__ void stage_x_i8_team(Team& team, const void* x, int dtype, int K, const uint16_t* norm_w, float eps, int g0,
                                int ng, int M, int ncols, const I8X& t) {
    const int nt = team.size(), tid = team.rank(), lane = tid & 31;
    const bool normed = norm_w != nullptr;
    const int upr_l = normed ? K / 8 : ng * 8;  // units per row read
    const int kfirst = normed ? 0 : g0 * kGroup;
    const int u0 = normed ? g0 * 8 : 0;         // first staged unit within a read row
    const int total_l = M * upr_l, per_chunk = kStageU * nt;
    const int nchunk = (total_l + per_chunk - 1) / per_chunk;
    float v[kStageU][8];
    uint4 nw[kStageU];
    auto load_chunk = [&](int c) {
#pragma unroll
        for (int u = 0; u < kStageU; ++u) {
            const int idx = c * per_chunk + u * nt + tid;
            if (idx < total_l) {
                const int k = kfirst + (idx % upr_l) * 8;
                load8(x, dtype, (int64_t)(idx / upr_l) * K + k, v[u]);
                if (normed) nw[u] = *reinterpret_cast<const uint4*>(norm_w + k);
            }
        }
    };
    load_chunk(0);
    STAGE_MARK(0);
    if (tid < M) t.amax[tid] = 0u;
    for (int i = tid; i < ng * ncols; i += nt) {
        t.xs[i] = 0.f;
        t.xe[i] = 0.f;
    }
    const int pad = ncols - 4 * M;
    for (int i = tid; i < ng * pad * 4; i += nt) {
        const int gl = i / (pad * 4), rem = i % (pad * 4);
        *reinterpret_cast<uint4*>(t.xq + ((size_t)gl * ncols + 4 * M + rem / 4) * 64 + (rem % 4) * 16) =
            make_uint4(0, 0, 0, 0);
    }
    team.sync();
    // norm sums per unit (reduced by finish_norm_factors in a fixed order) and raw row maxima:
    // max |x (1 + w)| with RMSNorm (the positive factor r scales the maximum afterwards; the
    // plane split only needs a bound within a factor of two), else max |x|
#pragma unroll 1
    for (int c = 0; c < nchunk; ++c) {
        if (c > 0) load_chunk(c);
#pragma unroll
        for (int u = 0; u < kStageU; ++u) {
            const int base = c * per_chunk + u * nt + tid - lane;  // warp-uniform
            if (base < total_l) {
                const int idx = base + lane;
                unsigned int bits = 0u;
                int m = -1;
                if (idx < total_l) {
                    m = idx / upr_l;
                    float amx = 0.f;
                    if (normed) {
                        t.ssq[idx] = unit_ssq(v[u], dtype);
                        const uint32_t w4[4] = {nw[u].x, nw[u].y, nw[u].z, nw[u].w};
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            amx = fmaxf(amx, fabsf(v[u][j] * (1.0f + bf16_bits_to_f32((w4[j >> 1] >> (16 * (j & 1))) & 0xffffu))));
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) amx = fmaxf(amx, fabsf(v[u][j]));
                    }
                    bits = __float_as_uint(amx);
                }
                warp_row_max(t.amax, bits, m, base, total_l, upr_l);
            }
        }
    }
    team.sync();
    STAGE_MARK(1);
    if (normed) norm_factors_team(team, dtype, M, K, eps, t.rf, t.ssq);  // ends with a barrier
    STAGE_MARK(2);
    for (int c = tid; c < ncols; c += nt) t.cs[c] = (c >> 2) < M ? pow2f(-10 - 7 * (c & 3)) : 0.f;
#pragma unroll 1
    for (int c = 0; c < nchunk; ++c) {
        if (nchunk > 1) load_chunk(c);
#pragma unroll
        for (int u = 0; u < kStageU; ++u) {
            const int base = c * per_chunk + u * nt + tid - lane;  // warp-uniform
            if (base < total_l) {
                const int idx = base + lane;
                const int m = idx < total_l ? idx / upr_l : 0, ul = idx < total_l ? idx % upr_l - u0 : -1;
                const bool ok = idx < total_l && ul >= 0 && ul < ng * 8;
                float s = 0.f, pe = 0.f;
                if (ok) {
                    if (normed) norm8(v[u], nw[u], t.rf[m]);
                    const float mx = normed ? __uint_as_float(t.amax[m]) * t.rf[m] * 1.001f : __uint_as_float(t.amax[m]);
                    const int e = row_exp(__float_as_uint(mx));
                    pe = pow2f(e);
                    uint32_t b[4][2];
                    planes8(v[u], e, b);
#pragma unroll
                    for (int j = 0; j < 8; ++j) s = __fadd_rn(s, v[u][j]);
                    const int gl = ul >> 3, u8 = ul & 7;
#pragma unroll
                    for (int p = 0; p < 4; ++p)
                        *reinterpret_cast<uint2*>(t.xq + ((size_t)gl * ncols + 4 * m + p) * 64 + u8 * 8) =
                            make_uint2(b[p][0], b[p][1]);
                }
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                s += __shfl_xor_sync(0xffffffffu, s, 4);
                if (ok && (lane & 7) == 0) {
                    const int o = (ul >> 3) * ncols + 4 * m;
                    t.xs[o] = __fmul_rn(s, 64.0f);
                    t.xe[o] = t.xe[o + 1] = t.xe[o + 2] = t.xe[o + 3] = pe;
                }
            }
        }
    }
    team.sync();
}

// Whole-block staging (the GEMV family and the lm_head kernel).
__device__ __forceinline__ void stage_x_i8(const void* x, int dtype, int K, const uint16_t* norm_w, float eps, int g0,
                                           int ng, int M, int ncols, const I8X& t) {
    BlockTeam team;
    stage_x_i8_team(team, x, dtype, K, norm_w, eps, g0, ng, M, ncols, t);
}

// bf16 value q (0..3) of four packed in a uint2, as binary32.
__device__ __forceinline__ float sel_bf16(uint2 v, int q) {
    const uint32_t w = q < 2 ? v.x : v.y;
    return __uint_as_float((q & 1) ? (w & 0xffff0000u) : (w << 16));
}

// ------------------------------------------------------------------------------------------------
// one stage (4 groups) of one warp's 16 rows: y[j][0..1] row g, y[j][2..3] row g+8, columns
// 8j + 2t + {0, 1} (lane = 4g + t).  A stage of ROWS rows holds the packed lines [ROWS][128 B],
// then the scales [ROWS][8 groups] and the biases [ROWS][8 groups].
// ------------------------------------------------------------------------------------------------
template <int NTN, int ROWS = 128, bool CHAIN = (NTN >= 2)>
__device__ __forceinline__ void i8_stage(const uint8_t* st, int so, int gl0, const I8X& t, int warp, int lane,
                                         float (&y)[NTN][4], float (&yb)[NTN][2]) {
    constexpr int ncols = 8 * NTN;  // activation columns (compile-time, so plane addresses fold)
    // plain loads (not volatile asm) so the compiler can hoist and interleave them across groups
    const int g = lane >> 2, tq = lane & 3;
    const int r0 = 16 * warp + g, r1 = r0 + 8;
    const uint8_t* sc = st + ROWS * 128;
    const uint8_t* bi = sc + ROWS * 16;
    const uint2 s0 = *reinterpret_cast<const uint2*>(sc + r0 * 16 + so);
    const uint2 s1 = *reinterpret_cast<const uint2*>(sc + r1 * 16 + so);
    const uint2 b0 = *reinterpret_cast<const uint2*>(bi + r0 * 16 + so);
    const uint2 b1 = *reinterpret_cast<const uint2*>(bi + r1 * 16 + so);
    uint2 wa[4], wb[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // the group's 32 bytes are units 2q, 2q+1 of the swizzled line
        const uint32_t off = (uint32_t)((((2 * q + (tq >> 1)) ^ g) << 4) + 8 * (tq & 1));
        wa[q] = *reinterpret_cast<const uint2*>(st + r0 * 128 + off);
        wb[q] = *reinterpret_cast<const uint2*>(st + r1 * 128 + off);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float sr0 = sel_bf16(s0, q), sr1 = sel_bf16(s1, q), br0 = sel_bf16(b0, q), br1 = sel_bf16(b1, q);
        const int gl = gl0 + q;
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            const uint4 xv = *reinterpret_cast<const uint4*>(t.xq + ((size_t)(gl * ncols + 8 * j + g) * 64 + 16 * tq));
            const int c0 = gl * ncols + 8 * j + 4 * (tq >> 1);  // plane-0 column of the lane's row
            if constexpr (CHAIN)
                i8_group_chained(wa[q], wb[q], xv, sr0, sr1, br0, br1, t.xe[c0], t.xs[c0], y[j], yb[j]);
            else
                i8_group(wa[q], wb[q], xv, sr0, sr1, br0, br1, t.xe[c0], t.xs[c0], y[j], yb[j]);
        }
    }
}


}  // namespace
}  // namespace marlin
