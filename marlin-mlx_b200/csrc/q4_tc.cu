// q4_tc.cu — tcgen05 (sm_100a) Q4 decode GEMV and fused lm_head + argmax.
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) for decode-sized
// activations (m * planes <= 32) of marlin-mlx (src/model/marlin.cpp:18-25, :31-35, :161-169) and
// the greedy mx::argmax after the lm_head (src/sampling/sampler.cpp:14-16).
//
// One CTA processes 128 weight rows at a time; TMEM lane i is weight row i:
//   * a producer thread streams the packed weights (2-D tensor map, [32 words x rows] boxes with
//     128-byte swizzle) and the scales/biases ([8 groups x rows] boxes) into a shared-memory ring;
//   * four dequant warps — thread = weight row — turn one 64-group of nibbles into bf16 (1 + q/16,
//     exact, one LOP3 per pair) and write it to TMEM with tcgen05.st (32 columns = the mma A tile
//     of 4 K16 steps), double-buffered;
//   * one thread issues tcgen05.mma (M=128, N=16/32, K=16; A from TMEM, B = the activation planes
//     from 128B-swizzled shared memory, D in TMEM per group) and tcgen05.commit;
//   * the dequant warps read the group's D (tcgen05.ld) and fold it in binary32:
//        y += 16*s*D + (b - 16*s)*sum_g(x)   ==  s*sum(x*q) + b*sum(x),
//     the reference's per-group dequant formula.
// The dequantized weights never touch shared memory, so shared-memory bandwidth stays far from
// the HBM rate, and the MMA runs on the tensor pipe while the CUDA cores dequantize the next group.
//
// tc_unit_kernel: one 128-row tile per thread-block cluster; the cluster's CTAs split K, their
// partial sums meet in the leader CTA through distributed shared memory; epilogue store / SwiGLU
// (64 gate + 64 up rows per tile) / residual add.  Weights are requested before
// griddepcontrol.wait.
// tc_lm_head_kernel: persistent over 128-row vocabulary tiles; the argmax is kept per thread as
// packed (ordered logit << 32 | ~index) keys, reduced per CTA and merged across CTAs with
// atomicMax; the last CTA decodes and re-zeroes the keys.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_stage.cuh"
#include "q4_host.cuh"
#include "q4_tc.cuh"

#include <cuda.h>

#include <algorithm>

namespace marlin {
namespace {

constexpr int kRows = 128;             // TMEM lanes = weight rows per tile
constexpr int kStageGroups = 8;        // 64-groups per ring stage (2 packed boxes)
constexpr uint32_t kBoxBytes = kRows * 128;  // [128 rows x 128 B]
constexpr uint32_t kStageBytes = 2 * kBoxBytes + 2 * kRows * 16;  // packed + scales + biases = 36 KB
constexpr int kThreads = 192;          // warps 0-3 dequant/fold, 4 TMA producer, 5 MMA + TMEM owner
constexpr uint32_t kTmemCols = 128;    // A: 2 x 32 columns, D: 2 x NCOL columns
// activation planes of one group: NCOL rows x 128 B (2 KB at NCOL = 16, 4 KB at 32)

// ------------------------------------------------------------------------------------------------
// activations as the mma B operand: [group][row][64 k] bf16, K-major, 128B swizzle, 8-row atoms;
// B row m*P + p holds plane p of activation row m (P = 1 for bf16, 3 for binary32 hi/mid/lo).
// Within each K16 step the k order is the fragment order {0,4,1,5,2,6,3,7, 8,12,...} so that it
// matches the nibble pairs (q_j, q_j+4) the dequant produces.
// ------------------------------------------------------------------------------------------------
struct TcX {
    uint8_t* xb;  // [ng][NCOL rows][128 B]
    float* xs;    // [ng][32] per-(group, plane row) sums
    float* rf;    // [M] RMSNorm factors
    float* ssq;   // [M*K/8] norm scratch
};

__device__ void stage_x_tc(const void* x, int dtype, int K, const uint16_t* norm_w, float eps, int g0, int ng,
                           int M, int P, int ncol, const TcX& t) {
    const int nt = blockDim.x, tid = threadIdx.x, lane = tid & 31;
    const int Meff = M * P;
    if (norm_w) {
        XGeom xg{nullptr, nullptr, t.rf, t.ssq, M, P, Meff, 0, 0};
        norm_factors_only(x, dtype, K, eps, xg);
    }
    // zero the padding rows [Meff, ncol) of every group
    const int padrows = ncol - Meff;
    for (int i = tid; i < ng * padrows * 8; i += nt) {
        const int gl = i / (padrows * 8), rem = i % (padrows * 8), r = Meff + rem / 8, u = rem % 8;
        *reinterpret_cast<uint4*>(t.xb + gl * ncol * 128 + r * 128 + u * 16) = make_uint4(0, 0, 0, 0);
    }
    const int upr = ng * 8, total = M * upr;
    const int k0 = g0 * kGroup;
    for (int base = tid - lane; base < total; base += nt) {  // warp-uniform trip count
        const int idx = base + lane;
        const bool ok = idx < total;
        const int m = ok ? idx / upr : 0, ul = ok ? idx % upr : 0;
        const int gl = ul >> 3, e0 = (ul & 7) * 8;  // group within the range, element within the group
        float v[8];
        float ps[3] = {0.f, 0.f, 0.f};
        if (ok) {
            const int k = k0 + ul * 8;
            load8(x, dtype, (int64_t)m * K + k, v);
            if (norm_w) {
                const uint4 nwv = *reinterpret_cast<const uint4*>(norm_w + k);
                const uint32_t w4[4] = {nwv.x, nwv.y, nwv.z, nwv.w};
                const float r = t.rf[m];
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
            const int u = 2 * (e0 >> 4) + ((e0 >> 3) & 1);  // 16-byte unit of the 128-byte row
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                if (p < P) {
                    const int r = m * P + p;
                    uint4 st;
                    st.x = pack_bf16x2(h[p][0], h[p][4]);
                    st.y = pack_bf16x2(h[p][1], h[p][5]);
                    st.z = pack_bf16x2(h[p][2], h[p][6]);
                    st.w = pack_bf16x2(h[p][3], h[p][7]);
                    *reinterpret_cast<uint4*>(t.xb + gl * ncol * 128 + r * 128 + ((u ^ (r & 7)) * 16)) = st;
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
                if (ok && (lane & 7) == 0) t.xs[gl * 32 + m * P + p] = s;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// shared pieces
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d_cta(void* dst, const CUtensorMap* tm, int32_t x, int32_t y, uint64_t* bar) {
    tma_load_2d(dst, tm, x, y, bar);
}

// Dequantize the 8 packed words of one group (this thread's row) into the 32 A-columns layout:
// K16 step s uses words 2s, 2s+1 -> columns 8s..8s+7 = q4_pairs(w[2s]), q4_pairs(w[2s+1]).
__device__ __forceinline__ void dequant_group(const uint8_t* line, int row, int g4, uint32_t (&a)[32]) {
    // the group's 32 bytes are 16-byte units 2*g4, 2*g4+1 of the (swizzled) 128-byte row line
    const uint4 lo = *reinterpret_cast<const uint4*>(line + (((2 * g4) ^ (row & 7)) * 16));
    const uint4 hi = *reinterpret_cast<const uint4*>(line + (((2 * g4 + 1) ^ (row & 7)) * 16));
    const uint32_t w[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t p[4];
        q4_pairs(w[j], p);
        a[4 * j + 0] = p[0];
        a[4 * j + 1] = p[1];
        a[4 * j + 2] = p[2];
        a[4 * j + 3] = p[3];
    }
}

// Compile-time shape of the activation block: NCOL mma columns (16 or 32), P planes per row,
// MFIX = exact row count (0: any m <= MS, checked at run time), LDC = TMEM columns read per fold.
template <int NCOL_, int P_, int MFIX_>
struct TcCfg {
    static constexpr int NCOL = NCOL_, P = P_, MFIX = MFIX_;
    static constexpr int MS = MFIX ? MFIX : NCOL / P;  // rows handled
    static constexpr int USED = MS * P;                // columns holding data
    static constexpr int LDC = USED <= 4 ? 4 : (USED <= 16 ? 16 : 32);
};

template <int LDC>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&d)[LDC]) {
    if (LDC == 4) {
        uint32_t r[4];
        tmem_ld4(taddr, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j % LDC] = __uint_as_float(r[j]);
    } else {
        uint32_t r[16];
        tmem_ld16(taddr, r);
        if (LDC == 32) {
            uint32_t r2[16];
            tmem_ld16(taddr + 16, r2);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) d[(j + 16) % LDC] = __uint_as_float(r2[j]);
        } else {
            tmem_wait_ld();
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) d[j % LDC] = __uint_as_float(r[j]);
    }
}

// (16 s, b - 16 s) of group gs (0..7) from the 8 scales / biases of a stage row (registers only).
__device__ __forceinline__ float2 stage_sb(uint4 sv, uint4 bv, int gs) {
    const int w = gs >> 1, sh = 16 * (gs & 1);
    const uint32_t s2 = w == 0 ? sv.x : (w == 1 ? sv.y : (w == 2 ? sv.z : sv.w));
    const uint32_t b2 = w == 0 ? bv.x : (w == 1 ? bv.y : (w == 2 ? bv.z : bv.w));
    const float sf = bf16_bits_to_f32((s2 >> sh) & 0xffffu), bf = bf16_bits_to_f32((b2 >> sh) & 0xffffu);
    return make_float2(sf * 16.0f, bf - sf * 16.0f);
}

// y[m*P + p] += 16 s * D + (b - 16 s) * sum over the first MS rows (MFIX or run-time M).
template <class C>
__device__ __forceinline__ void fold_group(float (&y)[C::USED], const float (&d)[C::LDC], const float* xs, float2 sb, int M) {
#pragma unroll
    for (int m = 0; m < C::MS; ++m) {
        if (C::MFIX || m < M) {
#pragma unroll
            for (int p = 0; p < C::P; ++p) {
                const int j = m * C::P + p;
                y[j] = fmaf(sb.x, d[j], fmaf(sb.y, xs[j], y[j]));
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// fused lm_head + argmax (persistent, one CTA per SM, all 512 TMEM columns)
//
// Warp roles (416 threads):
//   warps 0-7  dequant: warp w serves TMEM lane quarter w & 3 (rows 32(w&3) .. +31) and group
//              w >> 2 of each 2-group batch; after a named barrier over these 8 warps, one elected
//              thread issues the batch's 8 MMAs and commits them to d_ready[buf];
//   warps 8-11 fold: wait d_ready, read the two D blocks with tcgen05.ld, release the buffer
//              (d_free), apply scale and bias in binary32 and keep the running argmax keys;
//   warp 12    TMA producer for the stage ring.
// NB buffers of (2 x 32 A columns + 2 x NCOL D columns) rotate through TMEM, so up to 2 NB groups
// are between dequant and fold: enough to cover the MMA -> commit -> mbarrier latency.
// ------------------------------------------------------------------------------------------------
constexpr int kLmDeqWarps = 8;
constexpr int kLmThreads = (kLmDeqWarps + 4 + 1) * 32;
constexpr int kLmBatch = 2;  // 64-groups per MMA batch
constexpr uint32_t kLmTmemCols = 512;

template <class C>
struct LmBuf {
    static constexpr int ACOLS = kLmBatch * 32;
    static constexpr int DCOLS = kLmBatch * C::NCOL;
    static constexpr int NB = (int)kLmTmemCols / (ACOLS + DCOLS);  // 5 (NCOL 16) or 4 (NCOL 32)
    static constexpr int D0 = NB * ACOLS;                          // first D column
};

struct TcLmArgs {
    CUtensorMap tw, ts, tb;  // packed words [n][k/8] box [32 x 128]; scales, biases [n][k/64] box [8 x 128]
    LmHeadLaunch L;
    int P, Meff, G, S, ntiles;
    uint32_t off_ring, off_xb, off_xs, off_scr, off_bar, off_misc, off_sbq;
};

__device__ __forceinline__ unsigned long long logit_key(float v, int64_t idx) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <class C>
__global__ void __launch_bounds__(kLmThreads, 1) tc_lm_head_kernel(const __grid_constant__ TcLmArgs a) {
    using B = LmBuf<C>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const LmHeadLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G, S = a.S, M = (int)L.m;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* full = bars;             // [S]   TMA bytes landed
    uint64_t* empty = bars + S;        // [S]   8 dequant warps done with the stage
    uint64_t* d_ready = bars + 2 * S;  // [NB]  MMAs of the batch complete (+ issuer's arrive)
    uint64_t* d_free = d_ready + B::NB;  // [NB] 4 fold warps done with the buffer
    uint64_t* fin = d_free + B::NB;    // [1]   exit drain of the issuer's MMAs
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + a.off_misc);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc + 4);
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(smem + a.off_misc + 64);  // [4][M]
    float2* sbq = reinterpret_cast<float2*>(smem + a.off_sbq);  // [NB][2][128] (16 s, b - 16 s)
    uint8_t* ring = smem + a.off_ring;
    TcX tx{smem + a.off_xb, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_scr),
           reinterpret_cast<float*>(smem + a.off_scr) + 64};
    const int spt = G / kStageGroups;  // stages per tile (G % 8 == 0)
    const int bpt = G / kLmBatch;      // batches per tile
    const int my_tiles = a.ntiles > (int)blockIdx.x ? (a.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nstages = my_tiles * spt;
    const int nbatch = my_tiles * bpt;

    if (warp == 8) {
        tmem_alloc(tmem_slot, kLmTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kLmDeqWarps);
        }
        for (int b = 0; b < B::NB; ++b) {
            mbar_init(&d_ready[b], 2);
            mbar_init(&d_free[b], 4);
        }
        mbar_init(fin, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto issue_stage = [&](int q) {  // stage q of this CTA's sequence
        const int ti = q / spt, sp = q % spt;
        const int64_t row0 = (int64_t)(blockIdx.x + (int64_t)ti * gridDim.x) * kRows;
        const int gs = sp * kStageGroups;
        uint8_t* st = ring + (size_t)(q % S) * kStageBytes;
        mbar_arrive_expect_tx(&full[q % S], 2 * kBoxBytes + 2u * kRows * 16u);
        for (int c = 0; c < 2; ++c)
            tma_load_2d(st + c * kBoxBytes, &a.tw, (gs / 4 + c) * 32, (int32_t)row0, &full[q % S]);
        tma_load_2d(st + 2 * kBoxBytes, &a.ts, gs, (int32_t)row0, &full[q % S]);
        tma_load_2d(st + 2 * kBoxBytes + kRows * 16, &a.tb, gs, (int32_t)row0, &full[q % S]);
    };
    int issued = 0;
    if (warp == 12 && lane == 0) {
        prefetch_tmap(&a.tw);
        prefetch_tmap(&a.ts);
        prefetch_tmap(&a.tb);
        for (; issued < min(S, nstages); ++issued) issue_stage(issued);
    }
    pdl_wait();
    pdl_launch_dependents();
    stage_x_tc(L.x, L.x_dtype, (int)L.w.k, L.norm_w, L.eps, 0, G, M, C::P, C::NCOL, tx);
    fence_proxy_async_smem();  // activation planes (generic stores) -> tensor-core reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp == 12) {
        if (lane == 0) {
            for (; issued < nstages; ++issued) {
                const int q = issued;
                if (!thread_wait(&empty[q % S], (uint32_t)(((q / S) - 1) & 1), abort)) break;
                issue_stage(q);
            }
            // exit only once every copy this thread started has landed
            for (int q = max(0, issued - S); q < issued; ++q) drain_wait(&full[q % S], (uint32_t)((q / S) & 1));
        }
    } else if (warp < kLmDeqWarps) {
        const int quarter = warp & 3, gsub = warp >> 2;
        const int lrow = 32 * quarter + lane;
        const uint32_t lane_addr = (uint32_t)(32 * quarter) << 16;
        const uint32_t idesc = umma_idesc_bf16(kRows, C::NCOL);
        bool ok = true;
        for (int bi = 0; bi < nbatch; ++bi) {
            const int buf = bi % B::NB;
            const int ti = bi / bpt, gb = (bi % bpt) * kLmBatch;  // first group of the batch
            const int gl = gb + gsub;
            const int q = ti * spt + gl / kStageGroups;
            const int s = q % S, gs = gl % kStageGroups;
            if (ok && gs < kLmBatch) ok = warp_wait(&full[s], (uint32_t)((q / S) & 1), abort);
            if (ok && bi >= B::NB) ok = warp_wait(&d_free[buf], (uint32_t)(((bi / B::NB) - 1) & 1), abort);
            if (ok) {
                const uint8_t* st = ring + (size_t)s * kStageBytes;
                uint32_t av[32];
                dequant_group(st + (gs >> 2) * kBoxBytes + lrow * 128, lrow, gs & 3, av);
                const uint16_t sraw = *reinterpret_cast<const uint16_t*>(st + 2 * kBoxBytes + lrow * 16 + gs * 2);
                const uint16_t braw =
                    *reinterpret_cast<const uint16_t*>(st + 2 * kBoxBytes + kRows * 16 + lrow * 16 + gs * 2);
                const float sf = bf16_bits_to_f32(sraw), bfv = bf16_bits_to_f32(braw);
                sbq[(buf * kLmBatch + gsub) * kRows + lrow] = make_float2(sf * 16.0f, bfv - sf * 16.0f);
                tmem_st32(tmem + lane_addr + buf * B::ACOLS + gsub * 32, av);
                tmem_wait_st();
                if (gs >= kStageGroups - kLmBatch) {  // released once its words are in TMEM
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[s]);  // this warp no longer reads stage s
                }
            }
            tc_fence_before();
            named_bar_sync(1, kLmDeqWarps * 32);
            if (warp == 0 && lane == 0) {
                tc_fence_after();
                if (!*abort) {
#pragma unroll
                    for (int g = 0; g < kLmBatch; ++g) {
                        const uint8_t* xg = tx.xb + (gb + g) * (C::NCOL * 128);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            umma_tmem_a(tmem + B::D0 + buf * B::DCOLS + g * C::NCOL,
                                        tmem + buf * B::ACOLS + g * 32 + 8 * k, umma_desc_sw128(xg + 32 * k), idesc,
                                        k > 0);
                    }
                    umma_commit(&d_ready[buf]);
                }
                mbar_arrive(&d_ready[buf]);  // orders the sbq stores (named barrier above) before the fold
            }
        }
        if (warp == 0 && lane == 0) {  // every MMA this thread issued has completed before TMEM is freed
            umma_commit(fin);
            drain_wait(fin, 0);
        }
    } else {
        // fold warps: thread = row 32 * (warp & 3) + lane of the tile
        const int quarter = warp & 3;
        const int lrow = 32 * quarter + lane;
        const uint32_t lane_addr = (uint32_t)(32 * quarter) << 16;
        float y[C::USED];
        unsigned long long best = 0ull;  // lane m keeps the best key of activation row m
#pragma unroll
        for (int j = 0; j < C::USED; ++j) y[j] = 0.f;
        const bool bf16_logits = L.x_dtype == kBF16 && !L.norm_w;
        for (int bi = 0; bi < nbatch; ++bi) {
            const int buf = bi % B::NB;
            if (!warp_wait(&d_ready[buf], (uint32_t)((bi / B::NB) & 1), abort)) break;
            tc_fence_after();
            const int ti = bi / bpt, gb = (bi % bpt) * kLmBatch;
            const uint32_t dcol = tmem + lane_addr + B::D0 + buf * B::DCOLS;
            const float2 sb0 = sbq[(buf * kLmBatch + 0) * kRows + lrow];
            const float2 sb1 = sbq[(buf * kLmBatch + 1) * kRows + lrow];
            {
                float d[C::LDC];
                tmem_ld_cols<C::LDC>(dcol, d);
                fold_group<C>(y, d, tx.xs + gb * 32, sb0, M);
            }
            float d[C::LDC];
            tmem_ld_cols<C::LDC>(dcol + C::NCOL, d);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[buf]);
            fold_group<C>(y, d, tx.xs + (gb + 1) * 32, sb1, M);
            if (gb + kLmBatch == G) {  // tile finished: logits -> argmax keys (warp max per row)
                const int64_t row = (int64_t)(blockIdx.x + (int64_t)ti * gridDim.x) * kRows + lrow;
#pragma unroll
                for (int m = 0; m < C::MS; ++m) {
                    if (C::MFIX || m < M) {
                        float v = 0.f;
#pragma unroll
                        for (int p = 0; p < C::P; ++p) v += y[m * C::P + p];
                        if (bf16_logits) v = bf16_round(v);
                        unsigned long long k = row < L.w.n ? logit_key(v, L.vocab_offset + row) : 0ull;
#pragma unroll
                        for (int o = 16; o; o >>= 1) {
                            const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
                            k = other > k ? other : k;
                        }
                        if (lane == m) best = k > best ? k : best;
                    }
                }
#pragma unroll
                for (int j = 0; j < C::USED; ++j) y[j] = 0.f;
            }
        }
        if (lane < M) ckeys[quarter * M + lane] = best;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, kLmTmemCols);
    }
    __shared__ bool is_last;
    if (tid < M) {
        unsigned long long k = 0ull;
        for (int w = 0; w < 4; ++w) k = ckeys[w * M + tid] > k ? ckeys[w * M + tid] : k;
        if (k) atomicMax(&L.keys[tid], k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int prev = atomicAdd(L.counter, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        if (tid < M) {
            const unsigned long long k = atomicExch(&L.keys[tid], 0ull);
            if (L.keys_out) L.keys_out[tid] = k;
            const uint32_t o = (uint32_t)(k >> 32);
            const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
            if (L.ids) L.ids[tid] = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (L.best) L.best[tid] = __uint_as_float(u);
        }
        if (tid == 0) atomicExch(L.counter, 0u);
    }
}

// ------------------------------------------------------------------------------------------------
// decode GEMV: one 128-row tile per cluster, K split over the cluster's CTAs
// ------------------------------------------------------------------------------------------------
struct TcUnitArgs {
    CUtensorMap tw0, ts0, tb0, tw1, ts1, tb1;  // w0 (gate / main) and w1 (up) maps
    GemvLaunch L;
    int P, Meff, G, CL, gpc;  // gpc = groups per CTA
    uint32_t off_ring, off_xb, off_xs, off_scr, off_bar, off_misc, off_red;
};

template <class C, int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_unit_kernel(const __grid_constant__ TcUnitArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const GemvLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = (int)L.m, G = a.G, CL = a.CL;
    const uint32_t rank = CL > 1 ? cluster_rank() : 0u;
    const int tile = blockIdx.x / CL;
    const int g0 = (int)rank * a.gpc, ng = min(a.gpc, G - g0);
    const int nst = (ng + kStageGroups - 1) / kStageGroups;
    constexpr bool kSwiglu = EPI == kEpiSwiglu;
    constexpr int kHalf = kSwiglu ? kRows / 2 : kRows;  // rows per matrix in the tile
    const int64_t row0 = (int64_t)tile * kHalf;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* full = bars;            // [nst <= 8]
    uint64_t* a_full = bars + 8;      // [2]
    uint64_t* d_ready = a_full + 2;   // [2]
    uint64_t* d_free = d_ready + 2;   // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + a.off_misc);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc + 4);
    float* red = reinterpret_cast<float*>(smem + a.off_red);  // [CL][128 rows][USED]
    uint8_t* ring = smem + a.off_ring;
    TcX tx{smem + a.off_xb, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_scr),
           reinterpret_cast<float*>(smem + a.off_scr) + 64};

    if (warp == 5) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < nst; ++s) mbar_init(&full[s], 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&a_full[b], 4);
            mbar_init(&d_ready[b], 1);
            mbar_init(&d_free[b], 4);
        }
        fence_mbar_init();
        // all weights of this CTA's K range, before the dependency wait
        for (int s = 0; s < nst; ++s) {
            const int gs = g0 + s * kStageGroups, ngr = min(kStageGroups, g0 + ng - gs);
            const int nbox = (ngr + 3) / 4;
            uint8_t* st = ring + (size_t)s * kStageBytes;
            mbar_arrive_expect_tx(&full[s], nbox * kBoxBytes + 2u * kRows * 16u);
            for (int mtx = 0; mtx < (kSwiglu ? 2 : 1); ++mtx) {
                const CUtensorMap* tw = mtx ? &a.tw1 : &a.tw0;
                const CUtensorMap* ts = mtx ? &a.ts1 : &a.ts0;
                const CUtensorMap* tb = mtx ? &a.tb1 : &a.tb0;
                const uint32_t ro = mtx * kHalf;  // row offset of this matrix inside the tile
                for (int c = 0; c < nbox; ++c)
                    tma_load_2d(st + c * kBoxBytes + ro * 128, tw, (gs / 4 + c) * 32, (int32_t)row0, &full[s]);
                tma_load_2d(st + 2 * kBoxBytes + ro * 16, ts, gs, (int32_t)row0, &full[s]);
                tma_load_2d(st + 2 * kBoxBytes + kRows * 16 + ro * 16, tb, gs, (int32_t)row0, &full[s]);
            }
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    stage_x_tc(L.x, L.x_dtype, (int)L.w0.k, L.norm_w, L.eps, g0, ng, M, C::P, C::NCOL, tx);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    float y[C::USED];
#pragma unroll
    for (int j = 0; j < C::USED; ++j) y[j] = 0.f;
    const int lrow = 32 * (warp & 3) + lane;
    if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(kRows, C::NCOL);
            for (int gi = 0; gi < ng; ++gi) {
                const int buf = gi & 1;
                if (!thread_wait(&a_full[buf], (uint32_t)((gi >> 1) & 1), abort)) break;
                if (gi >= 2 && !thread_wait(&d_free[buf], (uint32_t)(((gi - 2) >> 1) & 1), abort)) break;
                tc_fence_after();
#pragma unroll
                for (int s = 0; s < 4; ++s)
                    umma_tmem_a(tmem + 64 + buf * C::NCOL, tmem + buf * 32 + 8 * s,
                                umma_desc_sw128(tx.xb + gi * (C::NCOL * 128) + 32 * s), idesc, s > 0);
                umma_commit(&d_ready[buf]);
            }
        }
    } else if (warp < 4) {
        const uint32_t lane_addr = (uint32_t)(32 * warp) << 16;
        float2 sb_prev = make_float2(0.f, 0.f);
        uint4 sv = make_uint4(0, 0, 0, 0), bv = make_uint4(0, 0, 0, 0);
        auto fold = [&](int gj, float2 sbj) -> bool {
            const int buf = gj & 1;
            if (!warp_wait(&d_ready[buf], (uint32_t)((gj >> 1) & 1), abort)) return false;
            tc_fence_after();
            float d[C::LDC];
            tmem_ld_cols<C::LDC>(tmem + lane_addr + 64 + buf * C::NCOL, d);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_free[buf]);
            fold_group<C>(y, d, tx.xs + gj * 32, sbj, M);
            return true;
        };
        bool ok = true;
        for (int gi = 0; gi < ng && ok; ++gi) {
            const int s = gi / kStageGroups, gs = gi % kStageGroups;
            const uint8_t* st = ring + (size_t)s * kStageBytes;
            if (gs == 0) {
                if (!warp_wait(&full[s], 0u, abort)) break;
                sv = *reinterpret_cast<const uint4*>(st + 2 * kBoxBytes + lrow * 16);
                bv = *reinterpret_cast<const uint4*>(st + 2 * kBoxBytes + kRows * 16 + lrow * 16);
            }
            uint32_t av[32];
            dequant_group(st + (gs >> 2) * kBoxBytes + lrow * 128, lrow, gs & 3, av);
            const float2 sb_cur = stage_sb(sv, bv, gs);
            const int buf = gi & 1;
            tmem_st32(tmem + lane_addr + buf * 32, av);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[buf]);
            if (gi >= 1) ok = fold(gi - 1, sb_prev);
            sb_prev = sb_cur;
        }
        if (ok && ng > 0) fold(ng - 1, sb_prev);
        // partial sums -> the leader's reduction buffer (slot = this CTA's rank)
        float* slot = red + ((size_t)rank * kRows + lrow) * C::USED;
#pragma unroll
        for (int j = 0; j < C::USED; ++j) {
            if (rank == 0) slot[j] = y[j];
            else st_cluster_f32(slot + j, 0, y[j]);
        }
    }
    tc_fence_before();
    if (CL > 1) cluster_sync_all();
    else __syncthreads();
    if (warp == 5) tmem_dealloc(tmem, kTmemCols);
    if (rank != 0 || warp >= 4) return;

    // leader epilogue: thread = tile row lrow; out[m] = sum over ranks and planes
    float o[C::MS];
#pragma unroll
    for (int m = 0; m < C::MS; ++m) {
        o[m] = 0.f;
        for (int r = 0; r < CL; ++r)
#pragma unroll
            for (int p = 0; p < C::P; ++p) o[m] += red[((size_t)r * kRows + lrow) * C::USED + m * C::P + p];
    }
    if (kSwiglu) {
        // up rows (lanes 64..127) hand their outputs to the gate rows through shared memory
        float* xch = red + (size_t)CL * kRows * C::USED;
        if (lrow >= kHalf) {
#pragma unroll
            for (int m = 0; m < C::MS; ++m) xch[(lrow - kHalf) * C::MS + m] = o[m];
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (lrow < kHalf) {
            const int64_t f = row0 + lrow;
            if (f < L.w0.n) {
#pragma unroll
                for (int m = 0; m < C::MS; ++m) {
                    if (C::MFIX || m < M) {
                        const float gsum = o[m], u = xch[lrow * C::MS + m];
                        if (L.y_dtype == kBF16) {
                            const float gq = bf16_round(gsum), uq = bf16_round(u);
                            const float sg = bf16_round(__fdividef(1.0f, 1.0f + expf(-gq)));
                            const float r = bf16_round(bf16_round(sg * gq) * uq);
                            static_cast<uint16_t*>(L.y)[(int64_t)m * L.ldy + f] = (uint16_t)f32_to_bf16_bits(r);
                        } else {
                            const float sg = 1.0f / (1.0f + expf(-gsum));
                            static_cast<float*>(L.y)[(int64_t)m * L.ldy + f] = (sg * gsum) * u;
                        }
                    }
                }
            }
        }
        return;
    }
    const int64_t row = row0 + lrow;
    if (row >= L.w0.n) return;
#pragma unroll
    for (int m = 0; m < C::MS; ++m) {
        if (C::MFIX || m < M) {
            float v = o[m];
            if (EPI == kEpiResid) {
                const float hv = L.resid_dtype == kBF16
                                     ? bf16_bits_to_f32(static_cast<const uint16_t*>(L.resid)[(int64_t)m * L.ldr + row])
                                     : static_cast<const float*>(L.resid)[(int64_t)m * L.ldr + row];
                v = hv + v;
            }
            if (L.y_dtype == kBF16)
                static_cast<uint16_t*>(L.y)[(int64_t)m * L.ldy + row] = (uint16_t)f32_to_bf16_bits(v);
            else
                static_cast<float*>(L.y)[(int64_t)m * L.ldy + row] = v;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
constexpr uint32_t kTcSmemLimit = 225 * 1024;
constexpr uint32_t kTcMinSmem = 80 * 1024;  // <= 2 TMEM-holding CTAs per SM (2 x 128 of 512 columns)

template <class C>
cudaError_t dispatch_tc_unit(const TcUnitArgs& a, int grid, int CL, uint32_t smem, int epi, bool pdl,
                             cudaStream_t stream) {
    if (epi == kEpiSwiglu) return launch_ex(tc_unit_kernel<C, kEpiSwiglu>, a, grid, kThreads, CL, smem, pdl, stream);
    if (epi == kEpiResid) return launch_ex(tc_unit_kernel<C, kEpiResid>, a, grid, kThreads, CL, smem, pdl, stream);
    return launch_ex(tc_unit_kernel<C, kEpiStore>, a, grid, kThreads, CL, smem, pdl, stream);
}

}  // namespace

bool tc_supported(int64_t k, int64_t m_eff) {
    return k % 512 == 0 && k >= 512 && m_eff >= 1 && m_eff <= 32 && tmap_encode_fn() != nullptr;
}

namespace {
uint32_t plan_tc_lm_head(const LmHeadLaunch& L, TcLmArgs& a, int& ncol);
uint32_t plan_tc_gemv(const GemvLaunch& L, TcUnitArgs& a, int& ncol, bool encode);
}  // namespace

bool tc_lm_head_fits(const LmHeadLaunch& L) {
    TcLmArgs a{};
    int ncol = 0;
    return plan_tc_lm_head(L, a, ncol) != 0;
}

bool tc_gemv_fits(const GemvLaunch& L) {
    TcUnitArgs a{};
    int ncol = 0;
    return plan_tc_gemv(L, a, ncol, false) != 0;
}

cudaError_t launch_tc_lm_head(const LmHeadLaunch& L, cudaStream_t stream) {
    TcLmArgs a{};
    int ncol = 0;
    const uint32_t smem = plan_tc_lm_head(L, a, ncol);
    if (!smem) return cudaErrorInvalidConfiguration;
    if (!encode_q4_maps(L.w, kRows, &a.tw, &a.ts, &a.tb)) return cudaErrorInvalidValue;
    const int grid = std::max(1, std::min(device_num_sms(), a.ntiles));
    if (a.P == 3) {
        if (L.m == 1) return launch_ex(tc_lm_head_kernel<TcCfg<16, 3, 1>>, a, grid, kLmThreads, 1, smem, L.pdl, stream);
        if (ncol == 16) return launch_ex(tc_lm_head_kernel<TcCfg<16, 3, 0>>, a, grid, kLmThreads, 1, smem, L.pdl, stream);
        return launch_ex(tc_lm_head_kernel<TcCfg<32, 3, 0>>, a, grid, kLmThreads, 1, smem, L.pdl, stream);
    }
    if (L.m == 1) return launch_ex(tc_lm_head_kernel<TcCfg<16, 1, 1>>, a, grid, kLmThreads, 1, smem, L.pdl, stream);
    if (ncol == 16) return launch_ex(tc_lm_head_kernel<TcCfg<16, 1, 0>>, a, grid, kLmThreads, 1, smem, L.pdl, stream);
    return launch_ex(tc_lm_head_kernel<TcCfg<32, 1, 0>>, a, grid, kLmThreads, 1, smem, L.pdl, stream);
}

cudaError_t launch_tc_gemv(const GemvLaunch& L, cudaStream_t stream) {
    TcUnitArgs a{};
    int ncol = 0;
    const uint32_t smem = plan_tc_gemv(L, a, ncol, true);
    if (!smem) return cudaErrorInvalidConfiguration;
    const int CL = a.CL;
    const int half = L.epi == kEpiSwiglu ? kRows / 2 : kRows;
    const int tiles = (int)((L.w0.n + half - 1) / half);
    const int grid = tiles * CL;
    if (a.P == 3) {
        if (L.m == 1) return dispatch_tc_unit<TcCfg<16, 3, 1>>(a, grid, CL, smem, L.epi, L.pdl, stream);
        if (ncol == 16) return dispatch_tc_unit<TcCfg<16, 3, 0>>(a, grid, CL, smem, L.epi, L.pdl, stream);
        return dispatch_tc_unit<TcCfg<32, 3, 0>>(a, grid, CL, smem, L.epi, L.pdl, stream);
    }
    if (L.m == 1) return dispatch_tc_unit<TcCfg<16, 1, 1>>(a, grid, CL, smem, L.epi, L.pdl, stream);
    if (ncol == 16) return dispatch_tc_unit<TcCfg<16, 1, 0>>(a, grid, CL, smem, L.epi, L.pdl, stream);
    return dispatch_tc_unit<TcCfg<32, 1, 0>>(a, grid, CL, smem, L.epi, L.pdl, stream);
}

namespace {

uint32_t plan_tc_lm_head(const LmHeadLaunch& L, TcLmArgs& a, int& ncol) {
    a.L = L;
    const int K = (int)L.w.k;
    a.G = K / kGroup;
    a.P = (L.norm_w || L.x_dtype == kF32) ? 3 : 1;
    a.Meff = (int)L.m * a.P;
    if (!tc_supported(K, a.Meff) || a.G % kStageGroups != 0) return 0;
    ncol = a.Meff <= 16 ? 16 : 32;
    const int nb = ncol == 16 ? LmBuf<TcCfg<16, 1, 0>>::NB : LmBuf<TcCfg<32, 1, 0>>::NB;
    a.ntiles = (int)((L.w.n + kRows - 1) / kRows);
    uint32_t off = 0;
    a.off_bar = off;
    off += 512;  // 2 S + 2 NB + 1 mbarriers (S <= 12)
    a.off_misc = off;
    off += 64 + 4 * 32 * 8;
    a.off_sbq = off;
    off += (uint32_t)nb * kLmBatch * kRows * 8;
    a.off_scr = off;
    off += align_up((64 + (L.norm_w ? (uint32_t)L.m * (K / 8) : 0u)) * 4, 128);
    a.off_xs = off;
    off += align_up((uint32_t)a.G * 32 * 4, 128);
    off = align_up(off, 1024);
    a.off_xb = off;
    off += (uint32_t)a.G * ncol * 128;
    a.off_ring = off;
    const uint32_t avail = kTcSmemLimit > off + 1024 ? kTcSmemLimit - off - 1024 : 0;
    a.S = std::min<int>(12, (int)(avail / kStageBytes));
    if (a.S < 2) return 0;
    return off + (uint32_t)a.S * kStageBytes + 1024;
}
uint32_t plan_tc_gemv(const GemvLaunch& L, TcUnitArgs& a, int& ncol, bool encode) {
    a.L = L;
    const int K = (int)L.w0.k;
    a.G = K / kGroup;
    a.P = (L.norm_w || L.x_dtype == kF32) ? 3 : 1;
    a.Meff = (int)L.m * a.P;
    if (!tc_supported(K, a.Meff)) return 0;
    ncol = a.Meff <= 16 ? 16 : 32;
    const bool swiglu = L.epi == kEpiSwiglu;
    const int half = swiglu ? kRows / 2 : kRows;
    const int tiles = (int)((L.w0.n + half - 1) / half);
    // cluster size: split K until the grid covers the SMs
    // (groups per CTA stay a multiple of 8: the scales box x-coordinate must be 16-byte aligned)
    int CL = 1;
    for (int c : {2, 4, 8}) {
        if ((int64_t)tiles * CL >= device_num_sms()) break;
        if (a.G % c == 0 && (a.G / c) % 8 == 0) CL = c;
    }
    if ((a.G / CL) % 8 != 0) return 0;
    a.CL = CL;
    a.gpc = a.G / CL;
    if (encode) {
        if (!encode_q4_maps(L.w0, half, &a.tw0, &a.ts0, &a.tb0)) return 0;
        if (swiglu && !encode_q4_maps(L.w1, half, &a.tw1, &a.ts1, &a.tb1)) return 0;
    }
    const int nst = (a.gpc + kStageGroups - 1) / kStageGroups;
    if (nst > 8) return 0;
    uint32_t off = 0;
    a.off_bar = off;
    off += 256;
    a.off_misc = off;
    off += 64;
    a.off_scr = off;
    off += align_up((64 + (L.norm_w ? (uint32_t)L.m * (K / 8) : 0u)) * 4, 128);
    a.off_xs = off;
    off += align_up((uint32_t)a.gpc * 32 * 4, 128);
    const int used = L.m == 1 ? a.P : ncol;  // data columns of the dispatched configuration
    a.off_red = off;
    off += align_up((uint32_t)(CL + 1) * kRows * used * 4, 128);  // partials + SwiGLU exchange
    off = align_up(off, 1024);
    a.off_xb = off;
    off += (uint32_t)a.gpc * ncol * 128;
    a.off_ring = off;
    off += (uint32_t)nst * kStageBytes;
    const uint32_t smem = std::max(off + 1024, kTcMinSmem);
    return smem <= kTcSmemLimit ? smem : 0;
}

}  // namespace

int tc_device_error(bool clear) { return tu_device_error(clear); }

}  // namespace marlin
