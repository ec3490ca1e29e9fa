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
//   * warp 5 (one thread) feeds the X ring, warp 9 (one thread) the weight and scale/bias rings
//     (separate warps: two producer loops in one warp serialise each other's waits);
//   * sixteen warps, two teams of eight taking alternate K steps, thread = weight row: dequantize one
//     group into bf16 W[256 x 64] in shared memory, K-major with 128-byte swizzle (the tcgen05
//     operand layout): per pair of codes one LOP3 (128 + q as bf16, exact), one FMA removing the
//     128 (exact) and one FMA q s + b (bf16x2, a single rounding), then PRMTs restore natural K
//     order; three buffers, so a team's fence and waits overlap the other
//     team's work;
//   * warp 1 (one thread): tcgen05.mma kind::f16 (bf16), M=128 N=256 K=16, A = X and B = W from
//     shared memory, D in TMEM (two 256-column accumulators, so the epilogue of one tile overlaps
//     the MMAs of the next);
//   * warps 12-15 and 23-26, two per TMEM lane quarter (each half of the columns): epilogue —
//     tcgen05.ld the accumulator (lane = activation row), then store
//     (bf16 / binary32), SwiGLU of a gate/up tile pair (128 gate + 128 up rows per tile) or a
//     residual add.
// Every wait is bounded (2 s): on timeout the kernel records a device error and drains.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_prefill.cuh"

#include <algorithm>

// Optional timeline hook, empty in the library build: PF_MARK(warp, lane, point, index) at phase
// boundaries of the MMA, dequant and epilogue loops (index = the CTA's running step or tile).
#ifndef PF_MARK
#define PF_MARK(w, l, k, i)
#endif

namespace marlin {
namespace {

constexpr int kPM = 128;                      // activation rows per MMA (M, TMEM lanes)
constexpr int kPN = 256;                      // weight rows per tile (MMA N)
constexpr uint32_t kPA = kPM * 128;           // X box: 128 rows x 64 bf16
constexpr uint32_t kPW = kPN * 32;            // packed words: 256 rows x 8 words
constexpr uint32_t kPSB = kPN * 16;           // scales (or biases): 256 rows x 8 groups
constexpr uint32_t kPB = kPN * 128;           // dequantized W: 256 rows x 64 bf16
constexpr int kPTeamWarps = 8;                // one dequant team: one thread per weight row
constexpr int kPDeqWarps = 2 * kPTeamWarps;   // two teams, alternate K steps
// Warp roles by warp index; warp w issues on SM sub-partition w % 4.  The MMA issuer (one thread that
// must keep the tensor pipe fed) shares its sub-partition with the two producers and two epilogue
// warps, which mostly sleep on barriers, and only two of the sixteen dequant warps; the other
// sub-partitions take two epilogue warps and four or five dequant warps each.
constexpr int kPWarpMma = 1, kPWarpX = 5, kPWarpW = 9;
constexpr int kPEpi0 = 12;                    // epilogue warps 12-15: TMEM lane quarters 0-3
constexpr int kPEpi1 = 23;                    // second epilogue set 23-26 (quarters 3, 0, 1, 2)
constexpr int kPEpiWarps = 8;
constexpr int kPThreads = (4 + kPDeqWarps + 3 + 4) * 32;

// dequant warp index 0..15 of a warp that has no other role
__device__ __forceinline__ int deq_index(int warp) {
    return warp - (warp > kPWarpMma) - (warp > kPWarpX) - (warp > kPWarpW) - (warp > kPEpi0 ? min(warp, kPEpi0 + 4) - kPEpi0 : 0);
}
constexpr uint32_t kPTmemCols = 512;
constexpr bool kPSleep = true;                // waiting threads sleep on the mbarrier (no spinning)

// Shared-memory plan for MH activation-row halves per tile (M = 128 MH): MH = 1 double-buffers the
// accumulator across tiles; MH = 2 uses both 256-column accumulators for one 256-row tile and so
// dequantizes each weight tile once for twice the MMA work (its epilogue then stalls the MMAs).
template <int MH>
struct PPlan {
    static constexpr int SX = MH == 1 ? 4 : 2;  // X ring stages
    static constexpr int SW = 6;                // packed-word ring stages
    static constexpr int NB = 3;                // dequantized W buffers
    static constexpr uint32_t XSTAGE = MH * kPA;
    static constexpr uint32_t OFF_W = SX * XSTAGE;
    static constexpr uint32_t OFF_SB = OFF_W + SW * kPW;
    static constexpr uint32_t OFF_B = OFF_SB + 2 * 2 * kPSB;
    static constexpr uint32_t OFF_BAR = OFF_B + NB * kPB;
    static constexpr uint32_t SMEM = 1024 + OFF_BAR + 512;
};

struct PrefillArgs {
    CUtensorMap tx, tw0, ts0, tb0, tw1, ts1, tb1;
    GemvLaunch L;
    int M, N, G;           // activation rows, output columns (features for SwiGLU), K groups
    int mtiles, ntiles;    // tile grid
    int vec;               // 1: y (and resid) rows allow 16-byte vector access at 16-column steps
};

__device__ __forceinline__ float swiglu_bf16(float g, float u) {
    const float gq = bf16_round(g), uq = bf16_round(u);
    const float sg = bf16_round(__fdividef(1.0f, 1.0f + expf(-gq)));
    return bf16_round(bf16_round(sg * gq) * uq);
}

// bf16x2 of (lo, hi), each rounded to nearest even
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

// swiglu_bf16 of two adjacent outputs, as bf16x2 (the first in the low half).  The same roundings:
// g, u and the sigmoid rounded to bf16 by cvt; each product of two bf16 values is exact in binary32,
// so one bf16 multiply (an FMA with -0) rounds it as bf16_round does.
__device__ __forceinline__ uint32_t swiglu_bf16x2(float g0, float g1, float u0, float u1) {
    constexpr uint32_t kNegZero2 = 0x80008000u;
    const uint32_t gq = cvt_bf16x2(g0, g1), uq = cvt_bf16x2(u0, u1);
    const float a0 = bf16_bits_to_f32(gq & 0xffffu), a1 = bf16_bits_to_f32(gq >> 16);
    const uint32_t sq = cvt_bf16x2(__fdividef(1.0f, 1.0f + expf(-a0)), __fdividef(1.0f, 1.0f + expf(-a1)));
    return bf16x2_fma(bf16x2_fma(sq, gq, kNegZero2), uq, kNegZero2);
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
    uint64_t* wfull = xempty + P::SX;     // [SW]
    uint64_t* wempty = wfull + P::SW;     // [SW] the warps of one dequant team
    uint64_t* sbfull = wempty + P::SW;    // [2]
    uint64_t* sbempty = sbfull + 2;       // [2] all dequant warps
    uint64_t* bfull = sbempty + 2;        // [NB] the warps of one dequant team
    uint64_t* bfree = bfull + P::NB;      // [NB] MMA commit
    uint64_t* dfull = bfree + P::NB;      // [2]
    uint64_t* dempty = dfull + 2;         // [2] 4 epilogue warps (per accumulator; per half when MH == 2)
    uint64_t* fin = dempty + 2;           // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int ntiles_total = a.mtiles * a.ntiles;
    const int my_tiles = ntiles_total > (int)blockIdx.x ? (ntiles_total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (warp == kPWarpMma) {
        tmem_alloc(tmem_slot, kPTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < P::SX; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&xempty[s], 1);
        }
        for (int s = 0; s < P::SW; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&wempty[s], kPTeamWarps);
        }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&sbfull[j], 1);
            mbar_init(&sbempty[j], kPDeqWarps);
            mbar_init(&dfull[j], 1);
            mbar_init(&dempty[j], kPEpiWarps);
        }
        for (int j = 0; j < P::NB; ++j) {
            mbar_init(&bfull[j], kPTeamWarps);
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

    if (warp == kPWarpX) {
        if (lane == 0) {  // X tiles
            prefetch_tmap(&a.tx);
            RingPos p;
            int issued = 0;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                int mt, nt;
                tile_coords(lt, mt, nt);
                for (int g = 0; g < G; ++g) {
                    if (p.round > 0 && !thread_wait<kPSleep>(&xempty[p.slot], (uint32_t)((p.round - 1) & 1), abort)) {
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
        }
    } else if (warp == kPWarpW) {
        if (lane == 0) {  // packed words, scales / biases
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
                        if (e >= 2 && !thread_wait<kPSleep>(&sbempty[se], (uint32_t)(((e >> 1) - 1) & 1), abort)) {
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
                    if (p.round > 0 && !thread_wait<kPSleep>(&wempty[p.slot], (uint32_t)((p.round - 1) & 1), abort)) {
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
                    p.next(P::SW);
                }
            }
            for (int q = max(0, issued - P::SW); q < issued; ++q) drain_wait(&wfull[q % P::SW], (uint32_t)((q / P::SW) & 1));
            for (int q = max(0, e - 2); q < e; ++q) drain_wait(&sbfull[q & 1], (uint32_t)((q >> 1) & 1));
        }
    } else if (warp == kPWarpMma) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(kPM, kPN);
            // operand descriptors of the ring bases; a stage, half or K slice at byte offset o adds
            // o >> 4 to the start-address field (addresses stay below 2^18, so the field never carries)
            const uint64_t xd0 = umma_desc_sw128(xring), bd0 = umma_desc_sw128(bbuf);
            RingPos px, pb;
            bool ok = true;
            for (int lt = 0; lt < my_tiles && ok; ++lt) {
                // MH == 1: accumulators alternate between tiles; MH == 2: both belong to every tile, and
                // half h is reused as soon as the epilogue has drained it (checked before its first MMA)
                const int acc = MH == 1 ? (lt & 1) : 0;
                if (MH == 1 && lt >= 2 && !thread_wait<kPSleep>(&dempty[acc], (uint32_t)(((lt >> 1) - 1) & 1), abort)) break;
                for (int g = 0; g < G; ++g) {
                    PF_MARK(warp, lane, 0, lt * G + g);
                    // both polls in flight at once (the common case: both stages are ready)
                    const bool xr = mbar_try_wait(&xfull[px.slot], (uint32_t)(px.round & 1));
                    const bool br = mbar_try_wait(&bfull[pb.slot], (uint32_t)(pb.round & 1));
                    if (!(xr && br) && (!thread_wait<kPSleep>(&xfull[px.slot], (uint32_t)(px.round & 1), abort) ||
                                        !thread_wait<kPSleep>(&bfull[pb.slot], (uint32_t)(pb.round & 1), abort))) {
                        ok = false;
                        break;
                    }
                    PF_MARK(warp, lane, 2, lt * G + g);
                    tc_fence_after();
                    const uint64_t xd = xd0 + (uint64_t)(((uint32_t)px.slot * P::XSTAGE) >> 4);
                    const uint64_t bd = bd0 + (uint64_t)(((uint32_t)pb.slot * kPB) >> 4);
#pragma unroll
                    for (int h = 0; h < MH; ++h) {
                        if (MH == 2 && g == 0 && lt >= 1) {
                            if (!thread_wait<kPSleep>(&dempty[h], (uint32_t)((lt - 1) & 1), abort)) {
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            umma_smem_a(tmem + (acc + h) * kPN, xd + (uint64_t)((h * kPA + 32 * k) >> 4),
                                        bd + (uint64_t)(2 * k), idesc, g > 0 || k > 0);
                    }
                    if (!ok) break;
                    PF_MARK(warp, lane, 3, lt * G + g);
                    umma_commit(&xempty[px.slot]);
                    umma_commit(&bfree[pb.slot]);
                    if (g == G - 1) umma_commit(&dfull[acc]);
                    px.next(P::SX);
                    pb.next(P::NB);
                }
            }
            umma_commit(fin);  // every MMA issued above completes before TMEM is released
            drain_wait(fin, 0);
        }
    } else if (warp < kPEpi0 || (warp >= kPEpi0 + 4 && warp < kPEpi1)) {
        // dequant: team tm takes the K steps of its parity (the two teams work on consecutive steps at
        // once); one thread per weight row n, its eight packed words of the group
        const int dw = deq_index(warp);
        const int tm = dw / kPTeamWarps;
        const int n = (dw % kPTeamWarps) * 32 + lane;
        const uint32_t rx = (uint32_t)(n & 7);  // 128-byte swizzle: 16-byte unit u of row n at (u ^ (n & 7)) * 16
        RingPos pw, pb;                         // positions of the CTA's running K step
        if (tm) {
            pw.next(P::SW);
            pb.next(P::NB);
        }
        int e = 0;
        bool ok = true;
        for (int lt = 0; lt < my_tiles && ok; ++lt) {
            for (int g = tm; g < G; g += 2) {  // G % 8 == 0: the parity of g is the parity of the step
                const int se = e & 1;
                PF_MARK(warp, lane, 0, lt * G + g);
                if ((g & 7) == tm && !warp_wait<kPSleep>(&sbfull[se], (uint32_t)((e >> 1) & 1), abort)) {
                    ok = false;
                    break;
                }
                if (!warp_wait<kPSleep>(&wfull[pw.slot], (uint32_t)(pw.round & 1), abort)) {
                    ok = false;
                    break;
                }
                PF_MARK(warp, lane, 1, lt * G + g);
                if (pb.round > 0 && !warp_wait<kPSleep>(&bfree[pb.slot], (uint32_t)((pb.round - 1) & 1), abort)) {
                    ok = false;
                    break;
                }
                PF_MARK(warp, lane, 2, lt * G + g);
                const uint8_t* ws = wring + (size_t)pw.slot * kPW + n * 32;
                const uint4 w0 = *reinterpret_cast<const uint4*>(ws);
                const uint4 w1 = *reinterpret_cast<const uint4*>(ws + 16);
                const uint8_t* sb = sbring + se * 2 * kPSB + n * 16 + (g & 7) * 2;
                const uint32_t sbits = *reinterpret_cast<const uint16_t*>(sb);
                const uint32_t bbits = *reinterpret_cast<const uint16_t*>(sb + kPSB);
                const uint32_t s2 = sbits | (sbits << 16), b2 = bbits | (bbits << 16);
                uint8_t* out = bbuf + (size_t)pb.slot * kPB + n * 128;
                const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    *reinterpret_cast<uint4*>(out + ((u ^ rx) << 4)) = dequant_word(wv[u], s2, b2);
                PF_MARK(warp, lane, 3, lt * G + g);
                fence_proxy_async_smem();  // generic stores -> visible to the tensor core
                __syncwarp();
                PF_MARK(warp, lane, 4, lt * G + g);
                const bool last = (g & 7) == 6 + tm;  // the team's last step on this scale/bias entry
                if (lane == 0) {
                    mbar_arrive(&wempty[pw.slot]);  // the packed words are consumed (dequantized and stored)
                    mbar_arrive(&bfull[pb.slot]);
                    if (last) mbar_arrive(&sbempty[se]);
                }
                if (last) ++e;
                pw.next(P::SW);
                pw.next(P::SW);
                pb.next(P::NB);
                pb.next(P::NB);
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
            PF_MARK(warp, lane, 0, lt);
            if (!warp_wait<kPSleep>(&dfull[acc], (uint32_t)(use & 1), abort)) break;
            PF_MARK(warp, lane, 1, lt);
            tc_fence_after();
            int mt, nt;
            tile_coords(lt, mt, nt);
            for (int h = 0; h < MH; ++h) {
                const int64_t m = ((int64_t)mt * MH + h) * kPM + 32 * quarter + lane;
                const bool row_ok = m < a.M;
                const uint32_t dcol = lane_base + (acc + h) * kPN;
                const int ncols = swiglu ? kPN / 2 : kPN;
                const int cbeg = warp >= kPEpi1 ? ncols / 2 : 0;  // two warps per lane quarter split the columns
                for (int c0 = cbeg; c0 < cbeg + ncols / 2; c0 += 16) {
                    uint32_t r0[16];
                    float v[16];
                    tmem_ld16(dcol + c0, r0);
                    if (swiglu) {
                        uint32_t u0[16];
                        tmem_ld16(dcol + kPN / 2 + c0, u0);
                        tmem_wait_ld();
                        if (ybf && row_ok && a.vec && (int64_t)nt * ncols + c0 + 16 <= a.N) {
                            uint32_t pk[8];
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                pk[i] = swiglu_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]),
                                                      __uint_as_float(u0[2 * i]), __uint_as_float(u0[2 * i + 1]));
                            uint4* yp = reinterpret_cast<uint4*>(static_cast<uint16_t*>(L.y) + m * L.ldy +
                                                                 (int64_t)nt * ncols + c0);
                            yp[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            yp[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                            continue;
                        }
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
                PF_MARK(warp, lane, 2 + h, lt);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kPWarpMma) {
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
