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
// Bounded wait that also ends early once another role has aborted (timeout recorded on device).
// Every lane acquires the barrier; the exit is warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity) ? 1 : 0)) return true;
        if ((it & 63u) == 63u) {
            int stop = 0;
            if ((threadIdx.x & 31) == 0) {
                if (*abort) {
                    stop = 1;
                } else if (globaltimer_ns() - t0 > 2000000000ull || it > (1u << 28)) {
                    record_device_error(kDevErrMbarTimeout);
                    *abort = 1;
                    stop = 1;
                }
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) return false;
        }
    }
}
// Single-thread bounded wait (producer / MMA issuer).
__device__ __forceinline__ bool thread_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0; it < (1u << 28); ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > 2000000000ull) {
                record_device_error(kDevErrMbarTimeout);
                *abort = 1;
                return false;
            }
        }
    }
    *abort = 1;
    return false;
}

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
// fused lm_head + argmax (persistent)
// ------------------------------------------------------------------------------------------------
struct TcLmArgs {
    CUtensorMap tw, ts, tb;  // packed words [n][k/8] box [32 x 128]; scales, biases [n][k/64] box [8 x 128]
    LmHeadLaunch L;
    int P, Meff, G, S, ntiles;
    uint32_t off_ring, off_xb, off_xs, off_scr, off_bar, off_misc;
};

__device__ __forceinline__ unsigned long long logit_key(float v, int64_t idx) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

template <class C>
__global__ void __launch_bounds__(kThreads, 1) tc_lm_head_kernel(const __grid_constant__ TcLmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const LmHeadLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G, S = a.S, M = (int)L.m;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* full = bars;            // [S]
    uint64_t* empty = bars + S;       // [S]
    uint64_t* a_full = bars + 2 * S;  // [2]
    uint64_t* d_ready = a_full + 2;   // [2]
    uint64_t* d_free = d_ready + 2;   // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + a.off_misc);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc + 4);
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(smem + a.off_misc + 64);  // [4][M]
    uint8_t* ring = smem + a.off_ring;
    TcX tx{smem + a.off_xb, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_scr),
           reinterpret_cast<float*>(smem + a.off_scr) + 64};
    const int spt = (G + kStageGroups - 1) / kStageGroups;  // stages per tile
    const int my_tiles = a.ntiles > (int)blockIdx.x ? (a.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nstages = my_tiles * spt;

    if (warp == 5) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&a_full[b], 4);
            mbar_init(&d_ready[b], 1);
            mbar_init(&d_free[b], 4);
        }
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto issue_stage = [&](int q) {  // stage q of this CTA's sequence
        const int ti = q / spt, sp = q % spt;
        const int64_t row0 = (int64_t)(blockIdx.x + (int64_t)ti * gridDim.x) * kRows;
        const int gs = sp * kStageGroups, ngr = min(kStageGroups, G - gs);
        uint8_t* st = ring + (size_t)(q % S) * kStageBytes;
        const int nbox = (ngr + 3) / 4;
        mbar_arrive_expect_tx(&full[q % S], nbox * kBoxBytes + 2u * kRows * 16u);
        for (int c = 0; c < nbox; ++c)
            tma_load_2d(st + c * kBoxBytes, &a.tw, (gs / 4 + c) * 32, (int32_t)row0, &full[q % S]);
        tma_load_2d(st + 2 * kBoxBytes, &a.ts, gs, (int32_t)row0, &full[q % S]);
        tma_load_2d(st + 2 * kBoxBytes + kRows * 16, &a.tb, gs, (int32_t)row0, &full[q % S]);
    };
    if (warp == 4 && lane == 0) {
        prefetch_tmap(&a.tw);
        prefetch_tmap(&a.ts);
        prefetch_tmap(&a.tb);
        for (int q = 0; q < min(S, nstages); ++q) issue_stage(q);
    }
    pdl_wait();
    pdl_launch_dependents();
    stage_x_tc(L.x, L.x_dtype, (int)L.w.k, L.norm_w, L.eps, 0, G, M, C::P, C::NCOL, tx);
    fence_proxy_async_smem();  // activation planes (generic stores) -> tensor-core reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    const int ngroups = my_tiles * G;
    if (warp == 4) {
        if (lane == 0) {
            for (int q = S; q < nstages; ++q) {
                if (!thread_wait(&empty[q % S], (uint32_t)(((q / S) - 1) & 1), abort)) break;
                issue_stage(q);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(kRows, C::NCOL);
            for (int gi = 0; gi < ngroups; ++gi) {
                const int buf = gi & 1;
                if (!thread_wait(&a_full[buf], (uint32_t)((gi >> 1) & 1), abort)) break;
                if (gi >= 2 && !thread_wait(&d_free[buf], (uint32_t)(((gi - 2) >> 1) & 1), abort)) break;
                tc_fence_after();
                const int gl = gi % G;
#pragma unroll
                for (int s = 0; s < 4; ++s)
                    umma_tmem_a(tmem + 64 + buf * C::NCOL, tmem + buf * 32 + 8 * s,
                                umma_desc_sw128(tx.xb + gl * (C::NCOL * 128) + 32 * s), idesc, s > 0);
                umma_commit(&d_ready[buf]);
            }
        }
    } else {
        // dequant / fold warps: thread = row 32*warp + lane of the tile
        const int lrow = 32 * warp + lane;
        const uint32_t lane_addr = (uint32_t)(32 * warp) << 16;
        float y[C::USED];
        unsigned long long best[C::MS];
#pragma unroll
        for (int j = 0; j < C::USED; ++j) y[j] = 0.f;
#pragma unroll
        for (int m = 0; m < C::MS; ++m) best[m] = 0ull;
        const bool bf16_logits = L.x_dtype == kBF16 && !L.norm_w;
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
            const int gl = gj % G;
            fold_group<C>(y, d, tx.xs + gl * 32, sbj, M);
            if (gl == G - 1) {  // tile finished: logits -> argmax keys
                const int64_t row = (int64_t)(blockIdx.x + (int64_t)(gj / G) * gridDim.x) * kRows + lrow;
                if (row < L.w.n) {
#pragma unroll
                    for (int m = 0; m < C::MS; ++m) {
                        if (C::MFIX || m < M) {
                            float v = 0.f;
#pragma unroll
                            for (int p = 0; p < C::P; ++p) v += y[m * C::P + p];
                            if (bf16_logits) v = bf16_round(v);
                            const unsigned long long k = logit_key(v, L.vocab_offset + row);
                            best[m] = k > best[m] ? k : best[m];
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < C::USED; ++j) y[j] = 0.f;
            }
            return true;
        };
        bool ok = true;
        for (int gi = 0; gi < ngroups && ok; ++gi) {
            const int ti = gi / G, gl = gi % G;
            const int q = ti * spt + gl / kStageGroups;
            const int s = q % S;
            const uint8_t* st = ring + (size_t)s * kStageBytes;
            const int gs = gl % kStageGroups;
            if (gs == 0) {
                if (!warp_wait(&full[s], (uint32_t)((q / S) & 1), abort)) break;
                sv = *reinterpret_cast<const uint4*>(st + 2 * kBoxBytes + lrow * 16);
                bv = *reinterpret_cast<const uint4*>(st + 2 * kBoxBytes + kRows * 16 + lrow * 16);
            }
            uint32_t av[32];
            dequant_group(st + (gs >> 2) * kBoxBytes + lrow * 128, lrow, gs & 3, av);
            const float2 sb_cur = stage_sb(sv, bv, gs);
            if (gs == kStageGroups - 1 || gl == G - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);  // this warp no longer reads stage s
            }
            const int buf = gi & 1;
            tmem_st32(tmem + lane_addr + buf * 32, av);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&a_full[buf]);
            if (gi >= 1) ok = fold(gi - 1, sb_prev);
            sb_prev = sb_cur;
        }
        if (ok && ngroups > 0) fold(ngroups - 1, sb_prev);
        // CTA reduction of the keys: warp max, then across the 4 dequant warps
#pragma unroll
        for (int m = 0; m < C::MS; ++m) {
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[m], o);
                best[m] = other > best[m] ? other : best[m];
            }
        }
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < C::MS; ++m)
                if (m < M) ckeys[warp * M + m] = best[m];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) tmem_dealloc(tmem, kTmemCols);
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

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(const float* local_ptr, uint32_t rank, float v) {
    uint32_t raddr;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(smem_u32(local_ptr)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(raddr), "f"(v) : "memory");
}

template <class C, int EPI>
__global__ void __launch_bounds__(kThreads, 1) tc_unit_kernel(const __grid_constant__ TcUnitArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tc_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool encode_maps(const Q4Mat& W, int box_rows, CUtensorMap* tw, CUtensorMap* ts, CUtensorMap* tb) {
    EncodeTiledFn fn = tc_encode_fn();
    if (!fn) return false;
    const cuuint32_t es[2] = {1, 1};
    {
        const cuuint64_t dims[2] = {(cuuint64_t)(W.k / 8), (cuuint64_t)W.n};
        const cuuint64_t strides[1] = {(cuuint64_t)(W.k / 2)};
        const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
        if (fn(tw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(W.w), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)(W.k / 64), (cuuint64_t)W.n};
    const cuuint64_t strides[1] = {(cuuint64_t)(W.k / 64 * 2)};
    const cuuint32_t box[2] = {8, (cuuint32_t)box_rows};
    for (int i = 0; i < 2; ++i) {
        if (fn(i ? tb : ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(i ? W.b : W.s), dims, strides, box,
               es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

int tc_num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

constexpr uint32_t kTcSmemLimit = 225 * 1024;
constexpr uint32_t kTcMinSmem = 80 * 1024;  // <= 2 TMEM-holding CTAs per SM (2 x 128 of 512 columns)

template <typename KernelT, typename ArgT>
cudaError_t tc_launch(KernelT kernel, const ArgT& args, int grid, int cluster, uint32_t smem, bool pdl,
                      cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

template <class C>
cudaError_t dispatch_tc_unit(const TcUnitArgs& a, int grid, int CL, uint32_t smem, int epi, bool pdl,
                             cudaStream_t stream) {
    if (epi == kEpiSwiglu) return tc_launch(tc_unit_kernel<C, kEpiSwiglu>, a, grid, CL, smem, pdl, stream);
    if (epi == kEpiResid) return tc_launch(tc_unit_kernel<C, kEpiResid>, a, grid, CL, smem, pdl, stream);
    return tc_launch(tc_unit_kernel<C, kEpiStore>, a, grid, CL, smem, pdl, stream);
}

}  // namespace

bool tc_supported(int64_t k, int64_t m_eff) {
    return k % 512 == 0 && k >= 512 && m_eff >= 1 && m_eff <= 32 && tc_encode_fn() != nullptr;
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
    if (!encode_maps(L.w, kRows, &a.tw, &a.ts, &a.tb)) return cudaErrorInvalidValue;
    const int grid = std::max(1, std::min(tc_num_sms(), a.ntiles));
    if (a.P == 3) {
        if (L.m == 1) return tc_launch(tc_lm_head_kernel<TcCfg<16, 3, 1>>, a, grid, 1, smem, L.pdl, stream);
        if (ncol == 16) return tc_launch(tc_lm_head_kernel<TcCfg<16, 3, 0>>, a, grid, 1, smem, L.pdl, stream);
        return tc_launch(tc_lm_head_kernel<TcCfg<32, 3, 0>>, a, grid, 1, smem, L.pdl, stream);
    }
    if (L.m == 1) return tc_launch(tc_lm_head_kernel<TcCfg<16, 1, 1>>, a, grid, 1, smem, L.pdl, stream);
    if (ncol == 16) return tc_launch(tc_lm_head_kernel<TcCfg<16, 1, 0>>, a, grid, 1, smem, L.pdl, stream);
    return tc_launch(tc_lm_head_kernel<TcCfg<32, 1, 0>>, a, grid, 1, smem, L.pdl, stream);
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
    if (!tc_supported(K, a.Meff)) return 0;
    ncol = a.Meff <= 16 ? 16 : 32;
    a.ntiles = (int)((L.w.n + kRows - 1) / kRows);
    uint32_t off = 0;
    a.off_bar = off;
    off += 256;
    a.off_misc = off;
    off += 64 + 4 * 32 * 8;
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
        if ((int64_t)tiles * CL >= tc_num_sms()) break;
        if (a.G % c == 0 && (a.G / c) % 8 == 0) CL = c;
    }
    if ((a.G / CL) % 8 != 0) return 0;
    a.CL = CL;
    a.gpc = a.G / CL;
    if (encode) {
        if (!encode_maps(L.w0, half, &a.tw0, &a.ts0, &a.tb0)) return 0;
        if (swiglu && !encode_maps(L.w1, half, &a.tw1, &a.ts1, &a.tb1)) return 0;
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

}  // namespace marlin
