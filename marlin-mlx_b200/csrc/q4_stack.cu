// q4_stack.cu — the whole Q4 decode step as one persistent cooperative kernel (sm_100a).
//
// Replaces, for decode-sized batches, the per-layer sequence of marlin-mlx's text model restricted
// to its Q4 sublayers (src/model/marlin.cpp:103-146: h += mlp(rms_norm(h)) with mlp_forward
// :31-35), the final norm (:145), the Q4 lm_head (:161-169) and the greedy argmax
// (src/sampling/sampler.cpp:14-16): one launch per token instead of 2 x layers + 1 dependent
// kernels (each dependent kernel boundary costs about 3 us on B200).
//
// All CTAs are resident (cooperative launch, one per SM).  Per layer:
//   phase A  work item = 16 features: the 16 gate rows and 16 up rows over K = hidden, SwiGLU in the
//            epilogue, binary32 act written to global memory;
//   phase B  work item = 32 rows of down_proj x 16 groups of K: a binary32 partial of h written to
//            part[chunk] (deterministic: no atomics);
// separated by software grid barriers among the consumer warps.  The next phase's staging forms
// h = h_prev + sum over chunks of part (fixed order), RMSNorms it and splits it into the exact s8
// planes of the integer-MMA path (see q4_i8.cu).  After the last layer the lm_head phase streams
// 32-row vocabulary items and keeps packed argmax keys.
//
// Warp roles: warps 0-7 consume (warp w: 16-row tile w & 1 of the item, 64-groups 2(w >> 1) and
// 2(w >> 1) + 1 of each 8-group stage; partial sums meet in shared memory at the end of the item);
// warp 8 is the TMA producer, which walks the same schedule across items, phases and layers, so
// the next phase's weights stream while the consumers wait at a grid barrier.
//
// Every wait is bounded: a grid barrier or mbarrier that does not complete within 2 s records a
// device error and raises an abort flag that every CTA checks, so all CTAs leave.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_i8_common.cuh"
#include "q4_stack.cuh"

#include <algorithm>

namespace marlin {
namespace {

constexpr int kSRows = 32;                         // weight rows per work item (two 16-row tiles)
constexpr int kSGroups = 8;                        // 64-groups per ring stage
constexpr uint32_t kSLine = kSRows * 128;          // one 4-group line box of 32 rows: 4 KB
constexpr uint32_t kSPacked = 2 * kSLine;          // 8 KB of packed words per stage
constexpr uint32_t kSSb = kSRows * 16;             // scales or biases: 8 groups x 32 rows
constexpr uint32_t kSStage = kSPacked + 2 * kSSb;  // 9 KB
constexpr int kSCons = 8;                          // consumer warps
constexpr int kSThreads = (kSCons + 1) * 32;
constexpr int kSBGroups = 16;                      // K groups per down-projection item
constexpr uint32_t kSSmemLimit = 225 * 1024;

// Bounded barrier among `n` warps built on an mbarrier (arrival count n): every lane of the warp
// waits for the phase; after 2 s (or once the CTA has aborted) it gives up, records `100 + where`
// and raises the CTA's abort flag, so no consumer can block forever.  `ph` is this warp's phase bit.
__device__ __forceinline__ void warp_group_bar(uint64_t* bar, uint32_t& ph, volatile int* abort, int where) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, ph) ? 1 : 0)) break;
        if ((it & 63u) == 63u) {
            int stop = 0;
            if ((threadIdx.x & 31) == 0 && (*abort || globaltimer_ns() - t0 > 2000000000ull)) {
                if (!*abort) record_device_error(100 + where);
                *abort = 1;
                stop = 1;
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) break;
        }
    }
    ph ^= 1u;
}

// the consumer warps (threads 0..255)
struct ConsumerTeam {
    uint64_t* bar;
    volatile int* abort;
    uint32_t ph = 0;
    int where = 0;
    __device__ __forceinline__ int size() const { return kSCons * 32; }
    __device__ __forceinline__ int rank() const { return threadIdx.x; }
    __device__ __forceinline__ void sync() { warp_group_bar(bar, ph, abort, where); }
};

struct StackLayerMaps {
    CUtensorMap g, gs, gb, u, us, ub, d, ds, db;
};

struct StackArgs {
    StackLayerMaps layer[kStackMaxLayers];
    CUtensorMap lw, ls, lb;
    const uint16_t* norm_w[kStackMaxLayers];
    const void* h0;
    int h0_dtype;
    const uint16_t* final_norm;
    float eps;
    int nl, M, H, I, GA, bchunks, ncols, S;
    int items_a, items_b, items_l;
    int64_t V;
    float* hbuf;  // [2][M][H] residual stream (binary32)
    float* act;   // [M][I]
    float* part;  // [bchunks][M][H] down-projection partials
    unsigned* bar;  // [0] arrivals, [1] generation, [2] abort, [3] CTAs finished
    unsigned long long* keys;  // [M] argmax keys (zero on entry, left zero)
    int32_t* ids;
    float* best;
    float* h_out;  // optional [M][H]: h before the final norm
    uint32_t off_bar, off_misc, off_ckeys, off_scr, off_xs, off_cs, off_xq, off_h, off_red, off_ring;
};

__device__ __forceinline__ unsigned long long stack_key(float v, int64_t idx) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

// Software grid barrier among the consumer warps of every CTA (all CTAs are co-resident by the
// cooperative launch).  The last arriver resets the arrival count and advances the generation.
// Returns false once any CTA has aborted (timeout anywhere).
__device__ bool grid_sync(ConsumerTeam& team, unsigned* bar, volatile int* abort) {
    team.where = 1;
    team.sync();
    if (threadIdx.x == 0 && !*abort) {
        volatile unsigned* gen = bar + 1;
        volatile unsigned* gabort = bar + 2;
        const unsigned g = *gen;
        __threadfence();
        if (atomicAdd(bar, 1u) == gridDim.x - 1) {
            atomicExch(bar, 0u);
            __threadfence();
            atomicAdd(bar + 1, 1u);
        } else {
            const uint64_t t0 = globaltimer_ns();
            while (*gen == g) {
                if (*gabort) {
                    *abort = 1;
                    break;
                }
                if (globaltimer_ns() - t0 > 2000000000ull) {
                    record_device_error(kDevErrMbarTimeout);
                    atomicExch(bar + 2, 1u);
                    *abort = 1;
                    break;
                }
                __nanosleep(32);
            }
        }
        __threadfence();
    }
    team.where = 2;
    team.sync();
    return !*abort;
}

// One 8-group stage of a 32-row item for consumer warp (tile t, groups 2kp, 2kp+1): the same
// tensor-core step as the decode GEMV (codes x s8 planes, exact int32, binary32 fold).
template <int NTN>
__device__ __forceinline__ void stack_stage(const uint8_t* st, int gl0, const I8X& t, int ncols, int tile, int kp,
                                            int lane, float (&y)[NTN][4]) {
    const int g = lane >> 2, tq = lane & 3;
    const int r0 = 16 * tile + g, r1 = r0 + 8;
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
        const int q = 2 * kp + qq;
        const int c = q >> 2, gq = q & 3;
        const uint32_t off = (uint32_t)((((2 * gq + (tq >> 1)) ^ g) << 4) + 8 * (tq & 1));
        const uint2 wa = *reinterpret_cast<const uint2*>(st + c * kSLine + r0 * 128 + off);
        const uint2 wb = *reinterpret_cast<const uint2*>(st + c * kSLine + r1 * 128 + off);
        const float sr0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + r0 * 16 + 2 * q));
        const float sr1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + r1 * 16 + 2 * q));
        const float br0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + kSSb + r0 * 16 + 2 * q));
        const float br1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + kSSb + r1 * 16 + 2 * q));
        const uint32_t a0[4] = {wa.x & kNib, wb.x & kNib, (wa.x >> 4) & kNib, (wb.x >> 4) & kNib};
        const uint32_t a1[4] = {wa.y & kNib, wb.y & kNib, (wa.y >> 4) & kNib, (wb.y >> 4) & kNib};
        const int gl = gl0 + q;
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            const uint4 xv = *reinterpret_cast<const uint4*>(t.xq + ((size_t)(gl * ncols + 8 * j + g) * 64 + 16 * tq));
            int cc[4] = {0, 0, 0, 0}, ee[4] = {0, 0, 0, 0};
            mma_s8_16832(cc, a0, xv.x, xv.y);
            mma_s8_16832(ee, a1, xv.z, xv.w);
            const float2 xs = *reinterpret_cast<const float2*>(t.xs + gl * ncols + 8 * j + 2 * tq);
            y[j][0] = fmaf(sr0, (float)(cc[0] + ee[0]), fmaf(br0, xs.x, y[j][0]));
            y[j][1] = fmaf(sr0, (float)(cc[1] + ee[1]), fmaf(br0, xs.y, y[j][1]));
            y[j][2] = fmaf(sr1, (float)(cc[2] + ee[2]), fmaf(br1, xs.x, y[j][2]));
            y[j][3] = fmaf(sr1, (float)(cc[3] + ee[3]), fmaf(br1, xs.y, y[j][3]));
        }
    }
}

template <int NTN>
__global__ void __launch_bounds__(kSThreads, 1) q4_stack_kernel(const __grid_constant__ StackArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int MS = 2 * NTN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = a.M, S = a.S, ncols = a.ncols, H = a.H, I = a.I, nb = (int)gridDim.x, cta = (int)blockIdx.x;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* empty = full + S;
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc);
    uint64_t* team_bars = reinterpret_cast<uint64_t*>(smem + a.off_misc + 16);  // [0] 8 consumers, [1] warps 0-1
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(smem + a.off_ckeys);  // [2][MS]
    float* hs = reinterpret_cast<float*>(smem + a.off_h);    // [M][H]
    float* red = reinterpret_cast<float*>(smem + a.off_red);  // [4][32][ncols], then [16][MS] exchange
    uint8_t* ring = smem + a.off_ring;
    I8X tx{smem + a.off_xq, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_cs),
           reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
           reinterpret_cast<unsigned int*>(smem + a.off_misc + 64)};
    const int spa = a.GA / kSGroups;         // stages per phase-A and lm_head item
    const int spb = kSBGroups / kSGroups;    // stages per phase-B item
    const int na = a.items_a > cta ? (a.items_a - 1 - cta) / nb + 1 : 0;
    const int nbi = a.items_b > cta ? (a.items_b - 1 - cta) / nb + 1 : 0;
    const int nli = a.items_l > cta ? (a.items_l - 1 - cta) / nb + 1 : 0;

    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSCons);
        }
        mbar_init(&team_bars[0], kSCons);
        mbar_init(&team_bars[1], 2);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kSCons) {
        // ---------------------------------------------------------------- producer (one thread)
        if (lane == 0) {
            int slot = 0, round = 0, issued = 0;
            bool ok = true;
            auto acquire = [&]() -> uint8_t* {
                if (round > 0 && !thread_wait(&empty[slot], (uint32_t)((round - 1) & 1), abort)) {
                    ok = false;
                    return nullptr;
                }
                mbar_arrive_expect_tx(&full[slot], kSStage);
                return ring + (size_t)slot * kSStage;
            };
            auto advance = [&]() {
                ++issued;
                if (++slot == S) {
                    slot = 0;
                    ++round;
                }
            };
            for (int l = 0; l < a.nl && ok; ++l) {
                const StackLayerMaps& mp = a.layer[l];
                for (int i = 0; i < na && ok; ++i) {
                    const int f0 = 16 * (cta + i * nb);
                    for (int s = 0; s < spa && ok; ++s) {
                        uint8_t* st = acquire();
                        if (!st) break;
                        const int gs = kSGroups * s;
                        for (int c = 0; c < 2; ++c) {
                            tma_load_2d(st + c * kSLine, &mp.g, (gs + 4 * c) * 8, f0, &full[slot]);
                            tma_load_2d(st + c * kSLine + kSLine / 2, &mp.u, (gs + 4 * c) * 8, f0, &full[slot]);
                        }
                        tma_load_2d(st + kSPacked, &mp.gs, gs, f0, &full[slot]);
                        tma_load_2d(st + kSPacked + kSSb / 2, &mp.us, gs, f0, &full[slot]);
                        tma_load_2d(st + kSPacked + kSSb, &mp.gb, gs, f0, &full[slot]);
                        tma_load_2d(st + kSPacked + kSSb + kSSb / 2, &mp.ub, gs, f0, &full[slot]);
                        advance();
                    }
                }
                for (int i = 0; i < nbi && ok; ++i) {
                    const int item = cta + i * nb, rb = item / a.bchunks, ch = item % a.bchunks;
                    for (int s = 0; s < spb && ok; ++s) {
                        uint8_t* st = acquire();
                        if (!st) break;
                        const int gs = kSBGroups * ch + kSGroups * s;
                        for (int c = 0; c < 2; ++c)
                            tma_load_2d(st + c * kSLine, &mp.d, (gs + 4 * c) * 8, kSRows * rb, &full[slot]);
                        tma_load_2d(st + kSPacked, &mp.ds, gs, kSRows * rb, &full[slot]);
                        tma_load_2d(st + kSPacked + kSSb, &mp.db, gs, kSRows * rb, &full[slot]);
                        advance();
                    }
                }
            }
            for (int i = 0; i < nli && ok; ++i) {
                const int item = cta + i * nb;
                for (int s = 0; s < spa && ok; ++s) {
                    uint8_t* st = acquire();
                    if (!st) break;
                    const int gs = kSGroups * s;
                    for (int c = 0; c < 2; ++c)
                        tma_load_2d(st + c * kSLine, &a.lw, (gs + 4 * c) * 8, kSRows * item, &full[slot]);
                    tma_load_2d(st + kSPacked, &a.ls, gs, kSRows * item, &full[slot]);
                    tma_load_2d(st + kSPacked + kSSb, &a.lb, gs, kSRows * item, &full[slot]);
                    advance();
                }
            }
            // exit only once every copy this thread started has landed
            for (int q = max(0, issued - S); q < issued; ++q) drain_wait(&full[q % S], (uint32_t)((q / S) & 1));
        }
    } else {
        // ---------------------------------------------------------------- consumers (warps 0-7)
        const int tile = warp & 1, kp = warp >> 1;
        const int g = lane >> 2, tq = lane & 3;
        ConsumerTeam team{&team_bars[0], abort};
        uint32_t ph2 = 0;  // phase of the warps 0-1 exchange barrier
        int slot = 0, round = 0;
        bool ok = true;
        unsigned long long best[NTN];
#pragma unroll
        for (int j = 0; j < NTN; ++j) best[j] = 0ull;

        // h = prev + sum of the down partials (fixed chunk order) into shared memory
        auto build_h = [&](const void* prev, int prev_dtype, float* hw) {
            const int n = M * H;
            for (int e = tid * 4; e < n; e += 256 * 4) {
                float4 v;
                if (prev_dtype == kBF16) {
                    const uint2 p = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(prev) + e);
                    v = make_float4(bf16_bits_to_f32(p.x & 0xffffu), bf16_bits_to_f32(p.x >> 16),
                                    bf16_bits_to_f32(p.y & 0xffffu), bf16_bits_to_f32(p.y >> 16));
                } else {
                    v = *reinterpret_cast<const float4*>(static_cast<const float*>(prev) + e);
                }
                for (int c = 0; c < a.bchunks; ++c) {
                    const float4 p = *reinterpret_cast<const float4*>(a.part + (size_t)c * n + e);
                    v.x += p.x;
                    v.y += p.y;
                    v.z += p.z;
                    v.w += p.w;
                }
                *reinterpret_cast<float4*>(hs + e) = v;
                if (hw) *reinterpret_cast<float4*>(hw + e) = v;
            }
            team.where = 3;
            team.sync();
        };
        // consume one item of nst stages starting at K group gl0 of the staged activations
        auto run_item = [&](int nst, int gl0, float (&y)[NTN][4]) {
#pragma unroll
            for (int j = 0; j < NTN; ++j) y[j][0] = y[j][1] = y[j][2] = y[j][3] = 0.f;
            for (int s = 0; s < nst; ++s) {
                if (ok && !warp_wait(&full[slot], (uint32_t)(round & 1), abort)) ok = false;
                if (ok) stack_stage<NTN>(ring + (size_t)slot * kSStage, gl0 + kSGroups * s, tx, ncols, tile, kp, lane, y);
#pragma unroll
                for (int j = 0; j < NTN; ++j) hold_regs(y[j]);  // the stage's data is consumed before release
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
                if (++slot == S) {
                    slot = 0;
                    ++round;
                }
            }
        };
        // partial sums of the 4 K-parts -> per (item row, activation row) outputs for warps 0-1:
        // returns, for lanes with (tq & 1) == 0, Y for rows 16*tile + g (ya) and + 8 (yb) and
        // activation row m = 2j + (tq >> 1)
        auto reduce_item = [&](const float (&y)[NTN][4], float (&ya)[NTN], float (&yb)[NTN]) {
#pragma unroll
            for (int j = 0; j < NTN; ++j) {
                const int col = 8 * j + 2 * tq;
                float* r0 = red + ((size_t)(kp * kSRows + 16 * tile + g) * ncols + col);
                float* r1 = r0 + 8 * ncols;
                r0[0] = y[j][0];
                r0[1] = y[j][1];
                r1[0] = y[j][2];
                r1[1] = y[j][3];
            }
            team.where = 4;
            team.sync();
            if (warp < 2) {
#pragma unroll
                for (int j = 0; j < NTN; ++j) {
                    const int col = 8 * j + 2 * tq;
                    float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
                    for (int k = 0; k < 4; ++k) {
                        const float* r0 = red + ((size_t)(k * kSRows + 16 * tile + g) * ncols + col);
                        const float* r1 = r0 + 8 * ncols;
                        t0 += r0[0];
                        t1 += r0[1];
                        t2 += r1[0];
                        t3 += r1[1];
                    }
                    const float2 cv = *reinterpret_cast<const float2*>(tx.cs + col);
                    float pa = fmaf(cv.x, t0, cv.y * t1), pb = fmaf(cv.x, t2, cv.y * t3);
                    pa += __shfl_xor_sync(0xffffffffu, pa, 1);
                    pb += __shfl_xor_sync(0xffffffffu, pb, 1);
                    ya[j] = pa;
                    yb[j] = pb;
                }
            }
            team.where = 5;
            team.sync();  // red is free again
        };

        const void* prev = a.h0;
        int prev_dtype = a.h0_dtype;
        for (int l = 0; l < a.nl; ++l) {
            // ---- phase A staging: x = RMSNorm(h) split into s8 planes (all GA groups)
            if (l == 0) {
                stage_x_i8_team(team, a.h0, a.h0_dtype, H, a.norm_w[0], a.eps, 0, a.GA, M, ncols, tx);
            } else {
                float* hw = a.hbuf + (size_t)(l & 1) * M * H;
                build_h(prev, prev_dtype, cta == 0 ? hw : nullptr);
                stage_x_i8_team(team, hs, kF32, H, a.norm_w[l], a.eps, 0, a.GA, M, ncols, tx);
                prev = hw;
                prev_dtype = kF32;
            }
            for (int i = 0; i < na; ++i) {
                float y[NTN][4], ya[NTN], yb[NTN];
                run_item(spa, 0, y);
                reduce_item(y, ya, yb);
                // SwiGLU of the 16 features: tile 0 rows are gate, tile 1 rows are up
                const int f0 = 16 * (cta + i * nb);
                if (warp == 1 && (tq & 1) == 0) {
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        const int m = 2 * j + (tq >> 1);
                        if (m < MS) {
                            red[g * MS + m] = ya[j];
                            red[(g + 8) * MS + m] = yb[j];
                        }
                    }
                }
                if (warp < 2) warp_group_bar(&team_bars[1], ph2, abort, 6);
                if (warp == 0 && (tq & 1) == 0) {
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        const int m = 2 * j + (tq >> 1);
                        if (m < M) {
                            const float ga = ya[j], gb = yb[j];
                            const float ua = red[g * MS + m], ub = red[(g + 8) * MS + m];
                            a.act[(size_t)m * I + f0 + g] = ((1.0f / (1.0f + expf(-ga))) * ga) * ua;
                            a.act[(size_t)m * I + f0 + g + 8] = ((1.0f / (1.0f + expf(-gb))) * gb) * ub;
                        }
                    }
                }
                if (warp < 2) warp_group_bar(&team_bars[1], ph2, abort, 7);
            }
            if (!grid_sync(team, a.bar, abort)) ok = false;
            // ---- phase B: down-projection partials, K chunk by chunk
            for (int i = 0; i < nbi; ++i) {
                const int item = cta + i * nb, rb = item / a.bchunks, ch = item % a.bchunks;
                stage_x_i8_team(team, a.act, kF32, I, nullptr, 0.f, kSBGroups * ch, kSBGroups, M, ncols, tx);
                float y[NTN][4], ya[NTN], yb[NTN];
                run_item(spb, 0, y);
                reduce_item(y, ya, yb);
                if (warp < 2 && (tq & 1) == 0) {
                    const int row = kSRows * rb + 16 * tile + g;
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        const int m = 2 * j + (tq >> 1);
                        if (m < M) {
                            float* pc = a.part + ((size_t)ch * M + m) * H;
                            pc[row] = ya[j];
                            pc[row + 8] = yb[j];
                        }
                    }
                }
            }
            if (!grid_sync(team, a.bar, abort)) ok = false;
        }
        // ---- final h, and the lm_head + argmax phase
        build_h(prev, prev_dtype, (cta == 0 && a.h_out) ? a.h_out : nullptr);
        if (a.items_l > 0) {
            stage_x_i8_team(team, hs, kF32, H, a.final_norm, a.eps, 0, a.GA, M, ncols, tx);
            for (int i = 0; i < nli; ++i) {
                const int item = cta + i * nb;
                float y[NTN][4], ya[NTN], yb[NTN];
                run_item(spa, 0, y);
                reduce_item(y, ya, yb);
                if (warp < 2) {
                    const int64_t rowa = (int64_t)kSRows * item + 16 * tile + g, rowb = rowa + 8;
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        const int m = 2 * j + (tq >> 1);
                        unsigned long long ka = (m < M && rowa < a.V) ? stack_key(ya[j], rowa) : 0ull;
                        const unsigned long long kb = (m < M && rowb < a.V) ? stack_key(yb[j], rowb) : 0ull;
                        ka = kb > ka ? kb : ka;
#pragma unroll
                        for (int o = 4; o < 32; o <<= 1) {
                            const unsigned long long other = __shfl_xor_sync(0xffffffffu, ka, o);
                            ka = other > ka ? other : ka;
                        }
                        best[j] = ka > best[j] ? ka : best[j];
                    }
                }
            }
            if (warp < 2 && g == 0 && (tq & 1) == 0) {
#pragma unroll
                for (int j = 0; j < NTN; ++j) ckeys[warp * MS + 2 * j + (tq >> 1)] = best[j];
            }
        }
        (void)ok;
    }
    __syncthreads();
    __shared__ bool is_last;
    if (a.items_l > 0 && tid < M) {
        const unsigned long long k = ckeys[tid] > ckeys[MS + tid] ? ckeys[tid] : ckeys[MS + tid];
        if (k) atomicMax(&a.keys[tid], k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int prevc = atomicAdd(a.bar + 3, 1u);
        is_last = (prevc == gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        if (a.items_l > 0 && tid < M) {
            const unsigned long long k = atomicExch(&a.keys[tid], 0ull);
            const uint32_t o = (uint32_t)(k >> 32);
            const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
            if (a.ids) a.ids[tid] = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (a.best) a.best[tid] = __uint_as_float(u);
        }
        if (tid == 0) {
            atomicExch(a.bar + 3, 0u);
            atomicExch(a.bar + 2, 0u);  // a timed-out call does not poison the next one
        }
    }
}

bool encode_rows(const Q4Mat& W, int rows, CUtensorMap* tw, CUtensorMap* ts, CUtensorMap* tb) {
    return encode_q4_maps(W, rows, tw, ts, tb);
}

}  // namespace

size_t stack_scratch_size(int64_t m, int64_t hidden, int64_t inter) {
    const int64_t bchunks = inter / 64 / kSBGroups;
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    return al((size_t)2 * m * hidden * 4) + al((size_t)m * inter * 4) + al((size_t)bchunks * m * hidden * 4);
}

bool stack_supported(int64_t m, int64_t hidden, int64_t inter, int n_layers) {
    return m >= 1 && m <= kStackMaxRows && n_layers >= 1 && n_layers <= kStackMaxLayers && hidden % 512 == 0 &&
           hidden <= 8192 && inter % (64 * kSBGroups) == 0 && inter % 512 == 0 && inter % 16 == 0 &&
           tmap_encode_fn() != nullptr;
}

cudaError_t launch_stack(const StackLaunch& L, cudaStream_t stream) {
    StackArgs a{};
    const int M = (int)L.m, H = (int)L.hidden, I = (int)L.inter;
    const int ntn = M <= 2 ? 1 : (M <= 4 ? 2 : 4);
    a.nl = L.n_layers;
    a.M = M;
    a.H = H;
    a.I = I;
    a.GA = H / 64;
    a.bchunks = I / 64 / kSBGroups;
    a.ncols = 8 * ntn;
    a.items_a = I / 16;
    a.items_b = (H / kSRows) * a.bchunks;
    a.items_l = L.lm ? (int)((L.lm->n + kSRows - 1) / kSRows) : 0;
    a.V = L.lm ? L.lm->n : 0;
    a.h0 = L.h0;
    a.h0_dtype = L.h0_dtype;
    a.final_norm = L.final_norm;
    a.eps = L.eps;
    for (int l = 0; l < a.nl; ++l) {
        const StackLayer& s = L.layers[l];
        a.norm_w[l] = s.norm;
        StackLayerMaps& mp = a.layer[l];
        if (!encode_rows(s.gate, 16, &mp.g, &mp.gs, &mp.gb) || !encode_rows(s.up, 16, &mp.u, &mp.us, &mp.ub) ||
            !encode_rows(s.down, kSRows, &mp.d, &mp.ds, &mp.db))
            return cudaErrorInvalidValue;
    }
    if (L.lm && !encode_rows(*L.lm, kSRows, &a.lw, &a.ls, &a.lb)) return cudaErrorInvalidValue;
    // scratch
    uint8_t* ws = static_cast<uint8_t*>(L.scratch);
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    a.hbuf = reinterpret_cast<float*>(ws);
    ws += al((size_t)2 * M * H * 4);
    a.act = reinterpret_cast<float*>(ws);
    ws += al((size_t)M * I * 4);
    a.part = reinterpret_cast<float*>(ws);
    a.bar = L.bar;
    a.keys = L.keys;
    a.ids = L.ids;
    a.best = L.best;
    a.h_out = L.h_out;
    // shared memory
    const int MS = 2 * ntn;
    uint32_t off = 0;
    auto take = [&](uint32_t bytes, uint32_t align) {
        off = (off + align - 1) / align * align;
        const uint32_t o = off;
        off += bytes;
        return o;
    };
    const uint32_t bars_bytes = 2 * 32 * 8;  // up to 32 stages
    a.off_bar = take(bars_bytes, 8);
    a.off_misc = take(128, 16);
    a.off_ckeys = take(2 * MS * 8, 16);
    a.off_scr = take((64 + (uint32_t)M * (H / 8)) * 4, 16);
    a.off_xs = take((uint32_t)a.GA * a.ncols * 4 * 2, 16);  // phase A / lm_head stage all of K; B stages 16 groups
    a.off_cs = take(a.ncols * 4, 16);
    a.off_xq = take((uint32_t)std::max(a.GA, kSBGroups) * a.ncols * 64, 128);
    a.off_h = take((uint32_t)M * H * 4, 16);
    a.off_red = take((uint32_t)4 * kSRows * a.ncols * 4 + 16 * MS * 4, 16);
    off = (off + 1023) / 1024 * 1024;
    a.off_ring = off;
    const uint32_t avail = kSSmemLimit > off + 1024 ? kSSmemLimit - off - 1024 : 0;
    a.S = std::min<int>(32, (int)(avail / kSStage));
    if (a.S < 4) return cudaErrorInvalidConfiguration;
    const uint32_t smem = off + (uint32_t)a.S * kSStage + 1024;
    const int grid = device_num_sms();

    auto go = [&](auto kernel) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kSThreads, smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kSThreads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kernel, a);
    };
    switch (ntn) {
        case 1: return go(q4_stack_kernel<1>);
        case 2: return go(q4_stack_kernel<2>);
        default: return go(q4_stack_kernel<4>);
    }
}

int stack_device_error(bool clear) { return tu_device_error(clear); }

}  // namespace marlin
