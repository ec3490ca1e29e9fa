// q4_prefill.cu — Q4 GEMM for prefill-sized activations on the 5th-generation tensor cores (sm_100a).
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) of marlin-mlx for
// many activation rows (the prefill call sites src/model/marlin.cpp:18-25, :31-35 with
// S ~ 2000 rows): y[m, n] = sum_k x[m, k] * w[n, k], bf16 x, binary32 accumulation, where each
// weight is dequantized once into the activation type, w = bf16(s q + b) with a single rounding —
// the way a quantized GEMM over many rows stages dequantized weight tiles in on-chip memory.
//
// One CTA owns a 128 (activation rows) x 256 (weight rows) output tile at a time (persistent over
// the tiles), K advancing one 64-group per step.  Three TMA rings, each released as soon as its
// consumer is done: X tiles [128 x 64] bf16 (128-byte swizzle; released by the MMA commit),
// packed words [256 rows x 8 words] (released by the dequant warps) and scales/biases
// [256 rows x 8 groups] (one entry per 8 groups).  Warp roles:
//   * warp 0: lane 0 feeds the X ring, lane 1 the weight and scale/bias rings;
//   * warps 2-9, thread = weight row: dequantize one group into bf16 W[256 x 64] in shared
//     memory, K-major with 128-byte swizzle (the tcgen05 operand layout): per pair of codes one
//     LOP3 (128 + q as bf16, exact), one FMA removing the 128 (exact) and one FMA q s + b (bf16x2,
//     a single rounding), then PRMTs restore natural K order; double-buffered;
//   * warp 1 (one thread): tcgen05.mma kind::f16 (bf16), M=128 N=256 K=16, A = X and B = W from
//     shared memory, D in TMEM (two 256-column accumulators, so the epilogue of one tile overlaps
//     the MMAs of the next);
//   * warps 10-13: epilogue — tcgen05.ld the accumulator (lane = activation row), then store
//     (bf16 / binary32), SwiGLU of a gate/up tile pair (128 gate + 128 up rows per tile) or a
//     residual add.
// Every wait is bounded (2 s): on timeout the kernel records a device error and drains.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_prefill.cuh"

#include <algorithm>

namespace marlin {
namespace {

constexpr int kPM = 128;                      // activation rows per MMA (M, TMEM lanes)
constexpr int kPN = 256;                      // weight rows per tile (MMA N)
constexpr int kPSW = 6;                       // packed-word ring stages
constexpr int kPNB = 2;                       // dequantized W buffers
constexpr uint32_t kPA = kPM * 128;           // X box: 128 rows x 64 bf16
constexpr uint32_t kPW = kPN * 32;            // packed words: 256 rows x 8 words
constexpr uint32_t kPSB = kPN * 16;           // scales (or biases): 256 rows x 8 groups
constexpr uint32_t kPB = kPN * 128;           // dequantized W: 256 rows x 64 bf16
constexpr int kPDeqWarps = 16;                // two threads per weight row
constexpr int kPThreads = (2 + kPDeqWarps + 4) * 32;  // producers, MMA, dequant, epilogue
constexpr uint32_t kPTmemCols = 512;

// Shared-memory plan for MH activation-row halves per tile (M = 128 MH): MH = 1 double-buffers the
// accumulator across tiles; MH = 2 uses both 256-column accumulators for one 256-row tile and so
// dequantizes each weight tile once for twice the MMA work.
template <int MH>
struct PPlan {
    static constexpr int SX = MH == 1 ? 5 : 3;  // X ring stages
    static constexpr uint32_t XSTAGE = MH * kPA;
    static constexpr uint32_t OFF_W = SX * XSTAGE;
    static constexpr uint32_t OFF_SB = OFF_W + kPSW * kPW;
    static constexpr uint32_t OFF_B = OFF_SB + 2 * 2 * kPSB;
    static constexpr uint32_t OFF_BAR = OFF_B + kPNB * kPB;
    static constexpr uint32_t SMEM = 1024 + OFF_BAR + 512;
};

struct PrefillArgs {
    CUtensorMap tx, tw0, ts0, tb0, tw1, ts1, tb1;
    GemvLaunch L;
    int M, N, G;           // activation rows, output columns (features for SwiGLU), K groups
    int mtiles, ntiles;    // tile grid
    int vec;               // 1: y (and resid) rows allow 16-byte vector access at 16-column steps
};

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Eight codes of one packed word -> eight bf16 weights s*q + b in natural K order (4 registers).
// LOP3 gives the pair (128 + q_i, 128 + q_i+4) as bf16 (exact), one FMA removes the 128 and one
// FMA forms q s + b with a single rounding; PRMTs regroup the pairs into K order 0..7.
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t s2, uint32_t b2) {
    constexpr uint32_t kOne2 = 0x3F803F80u, kNeg128 = 0xC300C300u, kMagic = 0x43004300u;
    uint32_t p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t v = lop3_and_or(w >> (4 * i), 0x000F000Fu, kMagic);
        p[i] = bf16x2_fma(bf16x2_fma(v, kOne2, kNeg128), s2, b2);  // (w_i, w_i+4)
    }
    uint4 o;
    o.x = __byte_perm(p[0], p[1], 0x5410);  // (w0, w1)
    o.y = __byte_perm(p[2], p[3], 0x5410);  // (w2, w3)
    o.z = __byte_perm(p[0], p[1], 0x7632);  // (w4, w5)
    o.w = __byte_perm(p[2], p[3], 0x7632);  // (w6, w7)
    return o;
}

__device__ __forceinline__ float swiglu_bf16(float g, float u) {
    const float gq = bf16_round(g), uq = bf16_round(u);
    const float sg = bf16_round(__fdividef(1.0f, 1.0f + expf(-gq)));
    return bf16_round(bf16_round(sg * gq) * uq);
}

// Ring position: slot and round advance together.
struct RingPos {
    int slot = 0, round = 0;
    __device__ __forceinline__ void next(int n) {
        if (++slot == n) {
            slot = 0;
            ++round;
        }
    }
};

template <int MH>
__global__ void __launch_bounds__(kPThreads, 1) q4_prefill_kernel(const __grid_constant__ PrefillArgs a) {
    using P = PPlan<MH>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const GemvLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G, epi = L.epi;
    const bool swiglu = epi == kEpiSwiglu;
    uint8_t* xring = smem;
    uint8_t* wring = smem + P::OFF_W;
    uint8_t* sbring = smem + P::OFF_SB;  // [2][scales 4 KB | biases 4 KB]
    uint8_t* bbuf = smem + P::OFF_B;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::OFF_BAR);
    uint64_t* xfull = bars;               // [SX]
    uint64_t* xempty = xfull + P::SX;     // [SX] MMA commit
    uint64_t* wfull = xempty + P::SX;     // [kPSW]
    uint64_t* wempty = wfull + kPSW;      // [kPSW] 8 dequant warps
    uint64_t* sbfull = wempty + kPSW;     // [2]
    uint64_t* sbempty = sbfull + 2;       // [2] 8 dequant warps
    uint64_t* bfull = sbempty + 2;        // [kPNB] 8 dequant warps
    uint64_t* bfree = bfull + kPNB;       // [kPNB] MMA commit
    uint64_t* dfull = bfree + kPNB;       // [2]
    uint64_t* dempty = dfull + 2;         // [2] 4 epilogue warps (per accumulator; per half when MH == 2)
    uint64_t* fin = dempty + 2;           // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int ntiles_total = a.mtiles * a.ntiles;
    const int my_tiles = ntiles_total > (int)blockIdx.x ? (ntiles_total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nsb = (G + 7) / 8;  // scale/bias entries per tile

    if (warp == 1) {
        tmem_alloc(tmem_slot, kPTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < P::SX; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], 1);
        }
        for (int s = 0; s < kPSW; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], kPDeqWarps);
        }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&sbfull[j], 1);
            mbar_init(&sbempty[j], kPDeqWarps);
            mbar_init(&dfull[j], 1);
            mbar_init(&dempty[j], 4);
        }
        for (int j = 0; j < kPNB; ++j) {
            mbar_init(&bfull[j], kPDeqWarps);
            mbar_init(&bfree[j], 1);
        }
        mbar_init(fin, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_launch_dependents();

    auto tile_coords = [&](int lt, int& mt, int& nt) {
        const int t = (int)blockIdx.x + lt * (int)gridDim.x;
        mt = t % a.mtiles;
        nt = t / a.mtiles;
    };

    if (warp == 0) {
        if (lane == 0) {  // X tiles
            prefetch_tmap(&a.tx);
            RingPos p;
            int issued = 0;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                int mt, nt;
                tile_coords(lt, mt, nt);
                for (int g = 0; g < G; ++g) {
                    if (p.round > 0 && !thread_wait(&xempty[p.slot], (uint32_t)((p.round - 1) & 1), abort)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&xfull[p.slot], P::XSTAGE);
#pragma unroll
                    for (int h = 0; h < MH; ++h)
                        tma_load_2d(xring + (size_t)p.slot * P::XSTAGE + h * kPA, &a.tx, g * 64, (mt * MH + h) * kPM,
                                    &xfull[p.slot]);
                    ++issued;
                    p.next(P::SX);
                }
            }
            for (int q = max(0, issued - P::SX); q < issued; ++q) drain_wait(&xfull[q % P::SX], (uint32_t)((q / P::SX) & 1));
        } else if (lane == 1) {  // packed words, scales / biases
            prefetch_tmap(&a.tw0);
            prefetch_tmap(&a.ts0);
            prefetch_tmap(&a.tb0);
            RingPos p;
            int issued = 0, e = 0;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                int mt, nt;
                tile_coords(lt, mt, nt);
                const int row0 = swiglu ? nt * (kPN / 2) : nt * kPN;
                for (int g = 0; g < G; ++g) {
                    if ((g & 7) == 0) {
                        const int se = e & 1;
                        if (e >= 2 && !thread_wait(&sbempty[se], (uint32_t)(((e >> 1) - 1) & 1), abort)) {
                            ok = false;
                            break;
                        }
                        uint8_t* sb = sbring + se * 2 * kPSB;
                        mbar_arrive_expect_tx(&sbfull[se], 2 * kPSB);
                        if (swiglu) {
                            tma_load_2d(sb, &a.ts0, g, row0, &sbfull[se]);
                            tma_load_2d(sb + kPSB / 2, &a.ts1, g, row0, &sbfull[se]);
                            tma_load_2d(sb + kPSB, &a.tb0, g, row0, &sbfull[se]);
                            tma_load_2d(sb + kPSB + kPSB / 2, &a.tb1, g, row0, &sbfull[se]);
                        } else {
                            tma_load_2d(sb, &a.ts0, g, row0, &sbfull[se]);
                            tma_load_2d(sb + kPSB, &a.tb0, g, row0, &sbfull[se]);
                        }
                        ++e;
                    }
                    if (p.round > 0 && !thread_wait(&wempty[p.slot], (uint32_t)((p.round - 1) & 1), abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sw = wring + (size_t)p.slot * kPW;
                    mbar_arrive_expect_tx(&wfull[p.slot], kPW);
                    if (swiglu) {
                        tma_load_2d(sw, &a.tw0, g * 8, row0, &wfull[p.slot]);
                        tma_load_2d(sw + kPW / 2, &a.tw1, g * 8, row0, &wfull[p.slot]);
                    } else {
                        tma_load_2d(sw, &a.tw0, g * 8, row0, &wfull[p.slot]);
                    }
                    ++issued;
                    p.next(kPSW);
                }
            }
            for (int q = max(0, issued - kPSW); q < issued; ++q) drain_wait(&wfull[q % kPSW], (uint32_t)((q / kPSW) & 1));
            for (int q = max(0, e - 2); q < e; ++q) drain_wait(&sbfull[q & 1], (uint32_t)((q >> 1) & 1));
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(kPM, kPN);
            RingPos px, pb;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                // MH == 1: accumulators alternate between tiles; MH == 2: both belong to every tile, and
                // half h is reused as soon as the epilogue has drained it (checked before its first MMA)
                const int acc = MH == 1 ? (lt & 1) : 0;
                if (MH == 1 && lt >= 2 && !thread_wait(&dempty[acc], (uint32_t)(((lt >> 1) - 1) & 1), abort)) break;
                for (int g = 0; g < G; ++g) {
                    if (!thread_wait(&xfull[px.slot], (uint32_t)(px.round & 1), abort) ||
                        !thread_wait(&bfull[pb.slot], (uint32_t)(pb.round & 1), abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint8_t* xa = xring + (size_t)px.slot * P::XSTAGE;
                    const uint8_t* wb = bbuf + (size_t)pb.slot * kPB;
#pragma unroll
                    for (int h = 0; h < MH; ++h) {
                        if (MH == 2 && g == 0 && lt >= 1) {
                            if (!thread_wait(&dempty[h], (uint32_t)((lt - 1) & 1), abort)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            umma_smem_a(tmem + (acc + h) * kPN, umma_desc_sw128(xa + h * kPA + 32 * k),
                                        umma_desc_sw128(wb + 32 * k), idesc, g > 0 || k > 0);
                    }
                    if (!ok) break;
                    umma_commit(&xempty[px.slot]);
                    umma_commit(&bfree[pb.slot]);
                    if (g == G - 1) umma_commit(&dfull[acc]);
                    px.next(P::SX);
                    pb.next(kPNB);
                }
            }
            umma_commit(fin);  // every MMA issued above completes before TMEM is released
            drain_wait(fin, 0);
        }
    } else if (warp < 2 + kPDeqWarps) {
        // dequant: two threads per weight row n, four packed words each
        const int t = tid - 64, n = t >> 1, half = t & 1;
        uint32_t uoff[4];  // 128-byte swizzle: 16-byte unit u of row n sits at (u ^ (n & 7)) * 16
#pragma unroll
        for (int i = 0; i < 4; ++i) uoff[i] = (uint32_t)(n * 128 + (((4 * half + i) ^ (n & 7)) << 4));
        RingPos pw, pb;
        int e = 0;
        bool ok = true;
        for (int lt = 0; lt < my_tiles && ok; ++lt) {
            for (int g = 0; g < G; ++g) {
                const int se = e & 1;
                if ((g & 7) == 0 && !warp_wait(&sbfull[se], (uint32_t)((e >> 1) & 1), abort)) {
                    ok = false;
                    break;
                }
                if (!warp_wait(&wfull[pw.slot], (uint32_t)(pw.round & 1), abort) ||
                    (pb.round > 0 && !warp_wait(&bfree[pb.slot], (uint32_t)((pb.round - 1) & 1), abort))) {
                    ok = false;
                    break;
                }
                const uint4 wq = *reinterpret_cast<const uint4*>(wring + (size_t)pw.slot * kPW + n * 32 + half * 16);
                const uint8_t* sb = sbring + se * 2 * kPSB + n * 16 + (g & 7) * 2;
                const uint32_t sbits = *reinterpret_cast<const uint16_t*>(sb);
                const uint32_t bbits = *reinterpret_cast<const uint16_t*>(sb + kPSB);
                const uint32_t s2 = sbits | (sbits << 16), b2 = bbits | (bbits << 16);
                uint8_t* out = bbuf + (size_t)pb.slot * kPB;
                *reinterpret_cast<uint4*>(out + uoff[0]) = dequant_word(wq.x, s2, b2);
                *reinterpret_cast<uint4*>(out + uoff[1]) = dequant_word(wq.y, s2, b2);
                *reinterpret_cast<uint4*>(out + uoff[2]) = dequant_word(wq.z, s2, b2);
                *reinterpret_cast<uint4*>(out + uoff[3]) = dequant_word(wq.w, s2, b2);
                fence_proxy_async_smem();  // generic stores -> visible to the tensor core
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&wempty[pw.slot]);  // the packed words are consumed (dequantized and stored)
                    mbar_arrive(&bfull[pb.slot]);
                    if ((g & 7) == 7 || g == G - 1) mbar_arrive(&sbempty[se]);
                }
                if ((g & 7) == 7 || g == G - 1) ++e;
                pw.next(kPSW);
                pb.next(kPNB);
            }
        }
    } else {
        // epilogue: TMEM lane quarter = warp & 3, lane = activation row within each 128-row half.
        // Each thread writes 16 consecutive columns of its row per step (16-byte stores).
        const int quarter = warp & 3;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * quarter) << 16);
        const bool ybf = L.y_dtype == kBF16;
        for (int lt = 0; lt < my_tiles; ++lt) {
            const int acc = MH == 1 ? (lt & 1) : 0;
            const int use = MH == 1 ? (lt >> 1) : lt;
            if (!warp_wait(&dfull[acc], (uint32_t)(use & 1), abort)) break;
            tc_fence_after();
            int mt, nt;
            tile_coords(lt, mt, nt);
            for (int h = 0; h < MH; ++h) {
                const int64_t m = ((int64_t)mt * MH + h) * kPM + 32 * quarter + lane;
                const bool row_ok = m < a.M;
                const uint32_t dcol = lane_base + (acc + h) * kPN;
                const int ncols = swiglu ? kPN / 2 : kPN;
                for (int c0 = 0; c0 < ncols; c0 += 16) {
                    uint32_t r0[16];
                    float v[16];
                    tmem_ld16(dcol + c0, r0);
                    if (swiglu) {
                        uint32_t u0[16];
                        tmem_ld16(dcol + kPN / 2 + c0, u0);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float g0 = __uint_as_float(r0[i]), x0 = __uint_as_float(u0[i]);
                            v[i] = ybf ? swiglu_bf16(g0, x0) : (g0 / (1.0f + expf(-g0))) * x0;
                        }
                    } else {
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r0[i]);
                    }
                    if (!row_ok) continue;
                    const int64_t col0 = (int64_t)nt * ncols + c0;
                    const bool full = a.vec && col0 + 16 <= a.N;
                    if (epi == kEpiResid) {
                        if (full && L.resid_dtype == kF32) {
                            const float4* rp = reinterpret_cast<const float4*>(static_cast<const float*>(L.resid) + m * L.ldr + col0);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float4 rv = rp[i];
                                v[4 * i] += rv.x;
                                v[4 * i + 1] += rv.y;
                                v[4 * i + 2] += rv.z;
                                v[4 * i + 3] += rv.w;
                            }
                        } else if (full) {
                            const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(L.resid) + m * L.ldr + col0);
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                const uint4 rv = rp[i];
                                const uint32_t w4[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    v[8 * i + 2 * j] += bf16_bits_to_f32(w4[j] & 0xffffu);
                                    v[8 * i + 2 * j + 1] += bf16_bits_to_f32(w4[j] >> 16);
                                }
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                if (col0 + i >= a.N) continue;
                                v[i] += L.resid_dtype == kBF16
                                            ? bf16_bits_to_f32(static_cast<const uint16_t*>(L.resid)[m * L.ldr + col0 + i])
                                            : static_cast<const float*>(L.resid)[m * L.ldr + col0 + i];
                            }
                        }
                    }
                    if (full && ybf) {
                        uint4* yp = reinterpret_cast<uint4*>(static_cast<uint16_t*>(L.y) + m * L.ldy + col0);
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            uint32_t p[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                p[j] = f32_to_bf16_bits(v[8 * i + 2 * j]) | (f32_to_bf16_bits(v[8 * i + 2 * j + 1]) << 16);
                            yp[i] = make_uint4(p[0], p[1], p[2], p[3]);
                        }
                    } else if (full) {
                        float4* yp = reinterpret_cast<float4*>(static_cast<float*>(L.y) + m * L.ldy + col0);
#pragma unroll
                        for (int i = 0; i < 4; ++i) yp[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            if (col0 + i >= a.N) continue;
                            if (ybf)
                                static_cast<uint16_t*>(L.y)[m * L.ldy + col0 + i] = (uint16_t)f32_to_bf16_bits(v[i]);
                            else
                                static_cast<float*>(L.y)[m * L.ldy + col0 + i] = v[i];
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&dempty[MH == 1 ? acc : h]);  // this accumulator half is drained
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kPTmemCols);
    }
}

}  // namespace

bool prefill_applies(const GemvLaunch& L) {
    if (L.m <= kPrefillMinRows || L.x_dtype != kBF16 || L.norm_w) return false;
    // k % 512: the scales/biases tensor maps need a 16-byte multiple row stride (k/64 * 2 bytes)
    if (L.w0.k % 512 != 0 || L.m > (int64_t)1 << 24) return false;
    if (L.epi == kEpiSwiglu && (L.w1.n != L.w0.n || L.w1.k != L.w0.k)) return false;
    return tmap_encode_fn() != nullptr;
}

cudaError_t launch_prefill(const GemvLaunch& L, cudaStream_t stream) {
    PrefillArgs a{};
    a.L = L;
    a.M = (int)L.m;
    a.N = (int)L.w0.n;
    a.G = (int)(L.w0.k / 64);
    const bool swiglu = L.epi == kEpiSwiglu;
    const int rows_per_tile = swiglu ? kPN / 2 : kPN;
    a.ntiles = (int)((L.w0.n + rows_per_tile - 1) / rows_per_tile);
    // 256-row tiles when they still give every SM about two tiles, else 128-row tiles
    const int mh = ((L.m + 2 * kPM - 1) / (2 * kPM)) * a.ntiles >= 2 * device_num_sms() ? 2 : 1;
    a.mtiles = (int)((L.m + mh * kPM - 1) / (mh * kPM));
    EncodeTiledFn fn = tmap_encode_fn();
    if (!fn) return cudaErrorInvalidValue;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)L.w0.k, (cuuint64_t)L.m};
        const cuuint64_t strides[1] = {(cuuint64_t)L.w0.k * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)kPM}, es[2] = {1, 1};
        if (fn(&a.tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(L.x), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    auto enc = [&](const Q4Mat& W, CUtensorMap* tw, CUtensorMap* ts, CUtensorMap* tb) -> bool {
        const cuuint32_t es[2] = {1, 1};
        const cuuint64_t wd[2] = {(cuuint64_t)(W.k / 8), (cuuint64_t)W.n};
        const cuuint64_t ws[1] = {(cuuint64_t)(W.k / 2)};
        const cuuint32_t wbox[2] = {8, (cuuint32_t)rows_per_tile};
        if (fn(tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(W.w), wd, ws, wbox, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
        const cuuint64_t sd[2] = {(cuuint64_t)(W.k / 64), (cuuint64_t)W.n};
        const cuuint64_t ss[1] = {(cuuint64_t)(W.k / 64 * 2)};
        const cuuint32_t sbox[2] = {8, (cuuint32_t)rows_per_tile};
        for (int i = 0; i < 2; ++i)
            if (fn(i ? tb : ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(i ? W.b : W.s), sd, ss, sbox,
                   es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return false;
        return true;
    };
    if (!enc(L.w0, &a.tw0, &a.ts0, &a.tb0)) return cudaErrorInvalidValue;
    if (swiglu && !enc(L.w1, &a.tw1, &a.ts1, &a.tb1)) return cudaErrorInvalidValue;
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    const size_t ysz = L.y_dtype == kBF16 ? 2 : 4, rsz = L.resid_dtype == kBF16 ? 2 : 4;
    a.vec = al16(L.y) && (L.ldy * (int64_t)ysz) % 16 == 0 &&
            (L.epi != kEpiResid || (al16(L.resid) && (L.ldr * (int64_t)rsz) % 16 == 0));
    const int tiles = a.mtiles * a.ntiles;
    const int grid = std::max(1, std::min(device_num_sms(), tiles));
    if (mh == 2) return launch_ex(q4_prefill_kernel<2>, a, grid, kPThreads, 1, PPlan<2>::SMEM, L.pdl, stream);
    return launch_ex(q4_prefill_kernel<1>, a, grid, kPThreads, 1, PPlan<1>::SMEM, L.pdl, stream);
}

int prefill_device_error(bool clear) { return tu_device_error(clear); }

}  // namespace marlin
