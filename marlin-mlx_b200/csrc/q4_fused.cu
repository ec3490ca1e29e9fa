// q4_fused.cu — the Q4 MLP layers of a decode step as one persistent kernel (sm_100a).
//
// Replaces, for decode-sized batches, the layer loop of marlin-mlx's text model restricted to its
// Q4 sublayers (src/model/marlin.cpp:103-146: per layer h += mlp_forward(rms_norm(h)), with
// rms_norm :12-16, swiglu :27-29, mlp_forward :31-35 and the qmatmul of :18-25 on every
// projection).  The final norm, lm_head and argmax follow as the fused lm_head kernel.
//
// Why one kernel.  At one activation row a layer streams 21 MB (3.3 us at HBM speed), but as two
// dependent launches it pays a launch boundary, a cluster reduction and an epilogue twice.  Here a
// layer waits once, on the words of its input h, and the weights of the next layer stream into
// shared memory while the current one finishes.
//
// Work split (inter = 64 G features, G CTAs, thread-block clusters of 8):
//   CTA c owns intermediate features [64 c, 64 c + 64): it computes their gate and up rows over all
//   of `hidden` from the exact s8 planes of h * (1 + w) (the integer-MMA arithmetic of q4_i8.cu;
//   the RMSNorm factor multiplies the row sums afterwards), then SwiGLU, and copies the 64
//   activations as s8 planes into the shared memory of the other seven CTAs of its cluster (bulk
//   copies over distributed shared memory, counted in bytes on one mbarrier per CTA).
//   CTA rank i of cluster j then multiplies down_proj rows [i hidden/8, (i+1) hidden/8) by the
//   cluster's 512 features (columns [512 j, 512 j + 512): one 16-byte scale box per row, fully
//   used) and adds the partial rows into the accumulator of the next h with integer atomics.
//
// Counted fixed point (poll_fix_rows): every accumulator word is (value * 2^27) << 5 plus a 5-bit count
// of the contributions added to it, each atomic add bringing +1.  The sum does not depend on the
// order of the adds (deterministic), and a word is complete when its count reaches the known number
// of contributions, so the next layer waits on the words themselves: no arrival counter, no
// release fence and no second round trip to read the data.  Cluster 0 also adds the residual h.
//
// Accumulators rotate over three buffers (acc_l = acc[l % 3]).  acc_{l+2} is zeroed, one slice per
// CTA, during layer l (complete words of acc_l prove that every CTA has read acc_{l-1}), followed
// by a fence before the CTA's own adds of layer l; acc_1 and acc_2 are zeroed at kernel start
// behind one arrival counter, which the next kernel clears.
//
// Warp roles: W consumer warps (8; the kernel also builds with 16, two warps per 16-row tile each
// taking two of a stage's four groups), which take the ring stages in pairs; the last warp is the TMA
// producer, which walks every layer's stages (gate/up: 64 + 64 rows x 4 groups; down_proj: up to 128
// rows x 4 groups; 20 KB each) through one ring, so the next layer's weights stream while the
// consumers wait for the current h.
//
// Every wait is bounded (SM clock cycles): one that runs out records a device error, raises the
// CTA's abort flag and the grid's abort word, and every other wait then returns at once; the CTAs
// leave through the closing cluster barrier.
#include "common.cuh"
#include "q4_fused.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_i8_common.cuh"
#include "q4_stage.cuh"

#include <algorithm>
#include <mutex>

// Optional timeline hooks, empty in the library build: FUSED_MARK(layer, point) at the phase
// boundaries of each layer, evaluated by every consumer thread (a definition keeps thread 0's);
// FUSED_PMARK(layer, point) in the producer thread when it issues a layer's first and last stage.
#ifndef FUSED_MARK
#define FUSED_MARK(l, k)
#endif
#ifndef FUSED_PMARK
#define FUSED_PMARK(l, k)
#endif
// FUSED_READY(l, ready): per warp and ring stage, whether the stage had landed when first polled.
#ifndef FUSED_READY
#define FUSED_READY(l, r)
#endif

namespace marlin {
namespace {

constexpr int kFCluster = 8;
constexpr int kFRows = 128;                         // rows per ring stage
constexpr uint32_t kFPacked = kFRows * 128;         // packed lines of one stage (4 groups per row)
constexpr uint32_t kFSb = kFRows * 16;              // scale (or bias) box: 8 groups x 128 rows
constexpr uint32_t kFStage = kFPacked + 2 * kFSb;   // 20 KB
constexpr uint32_t kFSmemLimit = 226 * 1024;
constexpr int kFBar = 1;                            // named barrier of the consumer warps
#ifndef FUSED_PAIRFOLD
#define FUSED_PAIRFOLD 1
#endif
// rows of h polled per round trip (more holds more words in registers: 4 spills at 8 rows)
#ifndef FUSED_POLL_ROWS
#define FUSED_POLL_ROWS 2
#endif
// one-tile fold of plane pairs (i8_group_pair): measured at one row 290.9 us per step against 293.2
constexpr bool kFPairFold = FUSED_PAIRFOLD != 0;

// Plane weights of the lane's two columns in the combine (the pair fold keeps one value per row).
template <bool CHAIN>
__device__ __forceinline__ float2 fold_weights(const float* cs, int j, int tq) {
    const float2 cv = *reinterpret_cast<const float2*>(cs + 8 * j + 2 * tq);
    if constexpr (!CHAIN && kFPairFold) return make_float2(cv.y, 0.f);
    return cv;
}

__host__ __device__ constexpr int fused_threads(int W) { return (W + 1) * 32; }

struct FusedLayerMaps {
    CUtensorMap g, gs, gb, u, us, ub, d, ds, db;  // gate/up boxes of 64 rows, down_proj boxes of RB rows
};

struct FusedArgs {
    FusedLayerMaps lay[kFusedMaxLayers];
    const uint16_t* norm_w[kFusedMaxLayers];
    const uint16_t* h0;
    unsigned long long* acc;
    unsigned* sync;
    unsigned long long wait_cycles;
    int M, H, n_layers, S;
    float eps;
    uint32_t off_bar, off_misc, off_hq, off_hxs, off_hxe, off_cs, off_aq, off_out, off_res, off_ring;
};
static_assert(sizeof(FusedArgs) <= 32000, "kernel parameters above the 32 KB limit");

// ---- counted fixed point, global synchronisation ------------------------------------------------------
// One contribution: round(v * 2^27) in the value field, +1 in the count field.
__device__ __forceinline__ unsigned long long fix_word(long long f) {
    return ((unsigned long long)f << kFixCountBits) + 1ull;
}
__device__ __forceinline__ long long to_fix(float v) { return __float2ll_rn(v * 134217728.0f); }

__device__ __forceinline__ void red_add_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Gives up a wait: records the timeout once, raises the grid's abort word and the CTA's flag.
__device__ __forceinline__ void give_up(unsigned* gabort, volatile int* abort) {
    record_device_error(kDevErrMbarTimeout);
    atomicExch(gabort, 1u);
    *abort = 1;
}

// Thread 0 of the consumers: wait until the start counter reaches `target`, bounded.
__device__ void grid_wait(unsigned* sync, unsigned target, unsigned long long limit, volatile int* abort) {
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 0;; ++it) {
        if (ld_relaxed(sync) >= target) {
            fence_acq_rel_gpu();
            return;
        }
        if ((it & 15u) == 15u) {
            if (ld_relaxed(sync + 1)) {
                *abort = 1;
                return;
            }
            if (cycles_now() - t0 > limit) {
                give_up(sync + 1, abort);
                return;
            }
        }
    }
}

__device__ __forceinline__ ulonglong2 ld_relaxed_v2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}

// Eight accumulator words of each of rows 0..M-1 (at p + m * stride), waited for until each holds
// `target` contributions (bounded; gives up on a timeout or an abort), as binary32.  The rows go in
// batches of FUSED_POLL_ROWS: every pending row's words of a batch are requested before any of them
// is checked, so a batch costs one round trip to L2 (8 rows: four, not eight).  The loads are relaxed;
// the fence after them gives the words acquire order (and with them the adders' earlier reads of
// the accumulator this CTA clears next).
template <int MS>
__device__ void poll_fix_rows(const unsigned long long* p, size_t stride, int M, unsigned target,
                              float (&v)[MS][8], unsigned* gabort, unsigned long long limit, volatile int* abort) {
    constexpr int PB = MS < FUSED_POLL_ROWS ? MS : FUSED_POLL_ROWS;
    unsigned long long t0 = 0;
    uint32_t it = 0;
#pragma unroll
    for (int b0 = 0; b0 < MS; b0 += PB) {
        unsigned pend = 0;
#pragma unroll
        for (int i = 0; i < PB; ++i)
            if (b0 + i < M) pend |= 1u << i;
        while (pend && !*abort) {
            ulonglong2 q[PB][4];
#pragma unroll
            for (int i = 0; i < PB; ++i) {
                if ((pend >> i) & 1u) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) q[i][k] = ld_relaxed_v2(p + (size_t)(b0 + i) * stride + 2 * k);
                }
            }
#pragma unroll
            for (int i = 0; i < PB; ++i) {
                if ((pend >> i) & 1u) {
                    bool done = true;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        done = done && ((unsigned)q[i][k].x & 31u) == target && ((unsigned)q[i][k].y & 31u) == target;
                    if (done) {
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            v[b0 + i][2 * k] = fix_value(q[i][k].x);
                            v[b0 + i][2 * k + 1] = fix_value(q[i][k].y);
                        }
                        pend &= ~(1u << i);
                    }
                }
            }
            if (!pend) break;
            if (it++ == 0) {
                t0 = cycles_now();
            } else if ((it & 7u) == 0u) {
                if (ld_relaxed(gabort)) {
                    *abort = 1;
                } else if (cycles_now() - t0 > limit) {
                    give_up(gabort, abort);
                }
            }
        }
    }
    fence_acq_rel_gpu();
}

// Named barrier of the consumer warps that also returns whether any of them passed `p` true: the
// abort decision is taken once per phase, identically in every consumer thread.
template <int W>
__device__ __forceinline__ bool cons_bar_or(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\t"
        "setp.ne.u32 pi, %1, 0;\n\t"
        "bar.red.or.pred po, %2, %3, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(kFBar), "r"(W * 32)
        : "memory");
    return r != 0;
}
template <int W>
__device__ __forceinline__ void cons_bar() {
    asm volatile("bar.sync %0, %1;" ::"r"(kFBar), "r"(W * 32) : "memory");
}

// Non-blocking test of an mbarrier phase (the timeline hook's readiness probe).
__device__ __forceinline__ __attribute__((unused)) bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// ---- distributed shared memory ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t mapa_u32(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
// Bulk copy of `bytes` (multiple of 16) from this CTA's shared memory to the cluster address dst,
// counted on the destination's mbarrier (cluster address bar).
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst, uint32_t src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "r"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Warp-wide bounded wait for the cluster's activation planes; gives up on a timeout, the CTA's abort
// flag or the grid's abort word.
__device__ bool warp_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned* gabort,
                                  unsigned long long limit) {
    if (__all_sync(0xffffffffu, mbar_try_wait_cluster(bar, parity) ? 1 : 0)) return true;
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 0;; ++it) {
        if (__all_sync(0xffffffffu, mbar_try_wait_cluster(bar, parity) ? 1 : 0)) return true;
        if ((it & 63u) == 63u) {
            int stop = 0;
            if ((threadIdx.x & 31) == 0) {
                if (*abort || ld_relaxed(gabort)) {
                    stop = 1;
                } else if (cycles_now() - t0 > limit) {
                    give_up(gabort, abort);
                    stop = 1;
                }
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) {
                *abort = 1;
                return false;
            }
        }
    }
}

// Zero this CTA's slice of an n-word accumulator (L2 only) with `nt` threads; true if any stored.
__device__ __forceinline__ bool zero_slice(unsigned long long* p, size_t n, int c, int G, int t, int nt) {
    const size_t b = n * (size_t)c / (size_t)G, e = n * (size_t)(c + 1) / (size_t)G;
    for (size_t i = b + t; i < e; i += nt) __stcg(p + i, 0ull);
    return b + t < e;
}

// i8_group with the lane's two plane columns folded as one integer, 128 D_p + D_{p+1} (exact, below
// 2^27), so each row takes one conversion and one fma per group instead of two; the pair's weight in
// the combine is that of plane p + 1.
__device__ __forceinline__ void i8_group_pair(uint2 wa, uint2 wb, uint4 xv, float sr0, float sr1, float br0, float br1,
                                              float xe, float x0, float (&y)[4], float (&yb)[2]) {
    const uint32_t lo[4] = {wa.x & kNib, wb.x & kNib, wa.y & kNib, wb.y & kNib};
    const uint32_t hi[4] = {wa.x & ~kNib, wb.x & ~kNib, wa.y & ~kNib, wb.y & ~kNib};
    int c[4] = {0, 0, 0, 0}, e[4] = {0, 0, 0, 0};
    mma_u8s8_16832(c, lo, xv.x, xv.z);  // even elements
    mma_u8s8_16832(e, hi, xv.y, xv.w);  // odd elements, times 16
    const int p0 = 128 * (16 * c[0] + e[0]) + (16 * c[1] + e[1]);
    const int p1 = 128 * (16 * c[2] + e[2]) + (16 * c[3] + e[3]);
    y[0] = fmaf(sr0 * xe, (float)p0, y[0]);
    y[2] = fmaf(sr1 * xe, (float)p1, y[2]);
    yb[0] = fmaf(br0, x0, yb[0]);
    yb[1] = fmaf(br1, x0, yb[1]);
}

// Activation operand in shared memory: per 64-group gl, the planes at xq + gl * qstride
// ([ncols][64] bytes), 64 x the group sums at xs[gl * xstride + column] and 2^e at xe[...].
struct FOperand {
    const uint8_t* xq;
    const float* xs;
    const float* xe;
    int qstride, xstride;
};

// One ring stage for a warp's 16-row tile rt, groups [q0, q0 + NQ) of the stage's four (see i8_stage
// in q4_i8_common.cuh for the layout and the arithmetic).
template <int NTN, int NQ, bool CHAIN>
__device__ __forceinline__ void f_stage(const uint8_t* st, int so, int gl0, int q0, const FOperand& t, int rt,
                                        int lane, float (&y)[NTN][4], float (&yb)[NTN][2]) {
    const int g = lane >> 2, tq = lane & 3;
    const int r0 = 16 * rt + g, r1 = r0 + 8;
    const uint8_t* sc = st + kFRows * 128;
    const uint8_t* bi = sc + kFRows * 16;
    const uint2 s0 = *reinterpret_cast<const uint2*>(sc + r0 * 16 + so);
    const uint2 s1 = *reinterpret_cast<const uint2*>(sc + r1 * 16 + so);
    const uint2 b0 = *reinterpret_cast<const uint2*>(bi + r0 * 16 + so);
    const uint2 b1 = *reinterpret_cast<const uint2*>(bi + r1 * 16 + so);
    uint2 wa[NQ], wb[NQ];
#pragma unroll
    for (int qq = 0; qq < NQ; ++qq) {
        const int q = NQ == 4 ? qq : q0 + qq;
        const uint32_t off = (uint32_t)((((2 * q + (tq >> 1)) ^ g) << 4) + 8 * (tq & 1));
        wa[qq] = *reinterpret_cast<const uint2*>(st + r0 * 128 + off);
        wb[qq] = *reinterpret_cast<const uint2*>(st + r1 * 128 + off);
    }
#pragma unroll
    for (int qq = 0; qq < NQ; ++qq) {
        const int q = NQ == 4 ? qq : q0 + qq;
        const float sr0 = sel_bf16(s0, q), sr1 = sel_bf16(s1, q), br0 = sel_bf16(b0, q), br1 = sel_bf16(b1, q);
        const int gl = gl0 + q;
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            const uint4 xv = *reinterpret_cast<const uint4*>(t.xq + (size_t)gl * t.qstride + (8 * j + g) * 64 + 16 * tq);
            const int c0 = gl * t.xstride + 8 * j + 4 * (tq >> 1);
            if constexpr (CHAIN)
                i8_group_chained(wa[qq], wb[qq], xv, sr0, sr1, br0, br1, t.xe[c0], t.xs[c0], y[j], yb[j]);
            else if constexpr (kFPairFold)
                i8_group_pair(wa[qq], wb[qq], xv, sr0, sr1, br0, br1, t.xe[c0], t.xs[c0], y[j], yb[j]);
            else
                i8_group(wa[qq], wb[qq], xv, sr0, sr1, br0, br1, t.xe[c0], t.xs[c0], y[j], yb[j]);
        }
    }
}

// ------------------------------------------------------------------------------------------------
// the kernel: NTN activation column tiles (2 rows each), W consumer warps
// ------------------------------------------------------------------------------------------------
template <int NTN, int W>
__global__ void __launch_bounds__(fused_threads(W), 1) fused_layers_kernel(const __grid_constant__ FusedArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    constexpr int MS = 2 * NTN;     // activation rows per pass (2 per 8-column MMA tile)
    constexpr int ncols = 8 * NTN;  // MMA columns: 4 planes per row
    constexpr int KP = W / 8;       // warps per 16-row tile (each takes 4 / KP groups of a stage)
    constexpr int NQ = 4 / KP;
    constexpr bool CHAIN = NTN >= 2;  // the packed fold pays off once the codes serve two column tiles
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rt = warp & 7, kp = warp >> 3;
    const int M = a.M, H = a.H, S = a.S, NL = a.n_layers;
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    const uint32_t crank = cluster_rank();
    const int cj = c / kFCluster;
    const unsigned target = (unsigned)(KP * (G / kFCluster));  // contributions per accumulator word
    const int HG = H / kGroup;                 // 64-groups of h
    const int RD = H / kFCluster;              // down_proj rows of this CTA
    const int rd0 = (int)crank * RD;
    const int RB = RD < kFRows ? RD : kFRows;  // rows per down_proj stage
    const int nhalf = RD / RB;
    const int gu_st = HG / 4;                  // gate/up stages per layer
    const int per_layer = gu_st + 2 * nhalf;
    const size_t MH = (size_t)M * H;

    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* empty = full + S;
    uint64_t* actbar = empty + S;  // [2]: activation planes of the cluster, by layer parity
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc);
    float* red = reinterpret_cast<float*>(smem + a.off_misc + 64);  // [W][MS] sums of squares
    uint8_t* hq = smem + a.off_hq;                                    // [HG][ncols][64] planes of h (1 + w)
    float* hxs = reinterpret_cast<float*>(smem + a.off_hxs);
    float* hxe = reinterpret_cast<float*>(smem + a.off_hxe);
    float* cs = reinterpret_cast<float*>(smem + a.off_cs);
    uint8_t* aq = smem + a.off_aq;  // [2 parities][8 slots]: activation planes [ncols][64], sums, exponents
    float* out = reinterpret_cast<float*>(smem + a.off_out);          // [KP][128][MS] gate / up rows
    float* res = reinterpret_cast<float*>(smem + a.off_res);          // [RD][MS] residual rows
    uint8_t* ring = smem + a.off_ring;
    constexpr uint32_t SB = (uint32_t)ncols * (64 + 8);  // one CTA's slot (copied as one piece)
    constexpr uint32_t aq_bytes = kFCluster * SB;
    float* xch = red + W * MS;  // [2][4][MS]: SwiGLU group maxima and sums of the two half-group warps

    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        mbar_init(&actbar[0], 1);  // own arrival (with the expected bytes of the seven peers' copies)
        mbar_init(&actbar[1], 1);
        fence_mbar_init();
    }
    // operand buffers start at zero (padding columns and the plane 1-3 sums are never written)
    for (int i = tid; i < HG * ncols * 4; i += fused_threads(W)) reinterpret_cast<uint4*>(hq)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < HG * ncols; i += fused_threads(W)) hxs[i] = hxe[i] = 0.f;
    for (int i = tid; i < (int)(2 * aq_bytes / 16); i += fused_threads(W))
        reinterpret_cast<uint4*>(aq)[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < ncols; i += fused_threads(W)) cs[i] = (i >> 2) < M ? pow2f(-10 - 7 * (i & 3)) : 0.f;
    __syncthreads();
    cluster_sync_all();  // peers' barriers and buffers are ready before any remote copy

    int armed = -1;  // consumers: last layer whose activation barrier was armed and not yet waited for
    if (warp == W) {
        // ---- TMA producer: every layer's stages in order through the ring ------------------------------
        pdl_launch_dependents();
        if (lane == 0) {
            int slot = 0, q = 0;
            uint32_t wrap = 0u;
            bool ok = true;
            for (int L = 0; L < NL && ok; ++L) {
                const FusedLayerMaps& mp = a.lay[L];
                for (int t = 0; t < per_layer; ++t) {
                    if (q >= S && !thread_wait(&empty[slot], wrap ^ 1u, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = ring + (size_t)slot * kFStage;
                    if (t == 0) FUSED_PMARK(L, 12);
                    if (t == per_layer - 1) FUSED_PMARK(L, 13);
                    if (t < gu_st) {  // gate rows 64c.. at rows 0-63 of the stage, up rows at 64-127
                        const int gs = 4 * t, y = 64 * c;
                        mbar_arrive_expect_tx(&full[slot], kFStage);
                        tma_load_2d(st, &mp.g, gs * 8, y, &full[slot]);
                        tma_load_2d(st + kFPacked, &mp.gs, gs & ~7, y, &full[slot]);
                        tma_load_2d(st + kFPacked + kFSb, &mp.gb, gs & ~7, y, &full[slot]);
                        tma_load_2d(st + 64 * 128, &mp.u, gs * 8, y, &full[slot]);
                        tma_load_2d(st + kFPacked + 64 * 16, &mp.us, gs & ~7, y, &full[slot]);
                        tma_load_2d(st + kFPacked + kFSb + 64 * 16, &mp.ub, gs & ~7, y, &full[slot]);
                    } else {  // down_proj rows rd0 + h RB .., groups 8 cj + 4 s ..
                        const int d = t - gu_st, h = d >> 1, s = d & 1;
                        const int gs = 8 * cj + 4 * s, y = rd0 + h * RB;
                        mbar_arrive_expect_tx(&full[slot], (uint32_t)RB * 160u);
                        tma_load_2d(st, &mp.d, gs * 8, y, &full[slot]);
                        tma_load_2d(st + kFPacked, &mp.ds, gs & ~7, y, &full[slot]);
                        tma_load_2d(st + kFPacked + kFSb, &mp.db, gs & ~7, y, &full[slot]);
                    }
                    ++q;
                    if (++slot == S) {
                        slot = 0;
                        wrap ^= 1u;
                    }
                }
            }
            // every issued stage has landed before the CTA may leave
            for (int r = std::max(0, q - S); r < q; ++r) drain_wait(&full[r % S], (uint32_t)((r / S) & 1));
        }
        __syncwarp();
    } else {
        // ---- consumers ---------------------------------------------------------------------------------
        pdl_wait();  // h0 and the cleared counter come from earlier kernels
        pdl_launch_dependents();
        const int units = H / 8;
        const bool has_unit = tid < units;  // thread t holds elements 8t..8t+7 of every row
        const int g = lane >> 2, tq = lane & 3;
        zero_slice(a.acc + MH, MH, c, G, tid, W * 32);
        zero_slice(a.acc + 2 * MH, MH, c, G, tid, W * 32);
        cons_bar<W>();
        if (tid == 0) red_release_add(a.sync, 1u);  // start arrival: acc_1, acc_2 cleared
        int slot = 0;
        uint32_t fpar = 0u;
        for (int L = 0; L < NL; ++L) {
            const int par = L & 1;
            uint4 nw = make_uint4(0, 0, 0, 0);
            if (has_unit) nw = *reinterpret_cast<const uint4*>(a.norm_w[L] + 8 * tid);
            const unsigned long long* accL = a.acc + (size_t)(L % 3) * MH;
            unsigned long long* accN = a.acc + (size_t)((L + 1) % 3) * MH;
            FUSED_MARK(L, 0);

            // ---- h_L (complete words) -> planes of h (1 + w) with per-group exponents; sums of squares --
            float v[MS][8];
#pragma unroll
            for (int m = 0; m < MS; ++m) {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[m][j] = 0.f;
                if (L == 0 && m < M && has_unit) load8(a.h0, kBF16, (int64_t)m * H + 8 * tid, v[m]);
            }
            if (L > 0 && has_unit) poll_fix_rows<MS>(accL + 8 * tid, (size_t)H, M, target, v, a.sync + 1, a.wait_cycles, abort);
            FUSED_MARK(L, 10);
            if (has_unit) {
                const int grp = tid >> 3, u8 = tid & 7;
                const bool resid_rows = cj == 0 && 8 * tid >= rd0 && 8 * tid < rd0 + RD;
#pragma unroll
                for (int m = 0; m < MS; ++m) {
                    if (m < M) {
                        const float ssq = unit_ssq(v[m], L == 0 ? kBF16 : kF32);
                        if (resid_rows) {
#pragma unroll
                            for (int j = 0; j < 8; ++j) res[(8 * tid - rd0 + j) * MS + m] = v[m][j];
                        }
                        const uint32_t w4[4] = {nw.x, nw.y, nw.z, nw.w};
                        float amx = 0.f, sm = 0.f;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            v[m][j] = __fmul_rn(v[m][j], __fadd_rn(1.0f, bf16_bits_to_f32((w4[j >> 1] >> (16 * (j & 1))) & 0xffffu)));
                            amx = fmaxf(amx, fabsf(v[m][j]));
                            sm = __fadd_rn(sm, v[m][j]);
                        }
                        unsigned bits = __float_as_uint(amx);
#pragma unroll
                        for (int o = 1; o < 8; o <<= 1) {
                            bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
                            sm += __shfl_xor_sync(0xffffffffu, sm, o);
                        }
                        const int e = row_exp(bits);
                        uint32_t b[4][2];
                        planes8(v[m], e, b);
#pragma unroll
                        for (int p = 0; p < 4; ++p)
                            *reinterpret_cast<uint2*>(hq + ((size_t)(grp * ncols + 4 * m + p) * 64 + 8 * u8)) =
                                make_uint2(b[p][0], b[p][1]);
                        if (u8 == 0) {
                            hxs[grp * ncols + 4 * m] = __fmul_rn(sm, 64.0f);
                            hxe[grp * ncols + 4 * m] = pow2f(e);
                        }
                        float sq = ssq;
#pragma unroll
                        for (int o = 16; o; o >>= 1) sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
                        if (lane == 0) red[warp * MS + m] = sq;
                    }
                }
            } else if (lane == 0) {
#pragma unroll
                for (int m = 0; m < MS; ++m) red[warp * MS + m] = 0.f;
            }
            if (cons_bar_or<W>(*abort != 0)) break;
            FUSED_MARK(L, 1);
            // RMSNorm row factor of row `lane` (lanes < M): r = 1/sqrt(mean(h^2) + eps), warps summed in order
            float rfl = 0.f;
            if (lane < M) {
                float s2 = 0.f;
                for (int w = 0; w < W; ++w) s2 = __fadd_rn(s2, red[w * MS + lane]);
                const float var = L == 0  // bf16 h0: MLX evaluates mean(square(x)) in bf16
                                      ? bf16_round(__fmul_rn(bf16_round(s2), bf16_round((float)(1.0 / (double)H))))
                                      : __fmul_rn(s2, (float)(1.0 / (double)H));
                rfl = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
            }

            // ---- gate / up rows of the CTA's 64 features over all of hidden -----------------------------
            const FOperand txh{hq, hxs, hxe, ncols * 64, ncols};
            float y[NTN][4], yb[NTN][2];
#pragma unroll
            for (int j = 0; j < NTN; ++j) y[j][0] = y[j][1] = y[j][2] = y[j][3] = yb[j][0] = yb[j][1] = 0.f;
            bool wok = true;
            // stages in pairs: both are waited for first, so each warp has eight groups of independent
            // MMAs to interleave, and both are released after their values are consumed
            for (int t = 0; t < gu_st; t += 2) {
                const int sa = slot;
                const uint32_t pa = fpar;
                if (++slot == S) {
                    slot = 0;
                    fpar ^= 1u;
                }
                const int sb = slot;
                const uint32_t pb = fpar;
                if (++slot == S) {
                    slot = 0;
                    fpar ^= 1u;
                }
                FUSED_READY(L, mbar_test_wait(&full[sa], pa) && mbar_test_wait(&full[sb], pb));
                if (wok) wok = warp_wait(&full[sa], pa, abort);
                if (wok) wok = warp_wait(&full[sb], pb, abort);
                if (t == 0) FUSED_MARK(L, 6);
                if (t == gu_st - 2) FUSED_MARK(L, 8);
                if (wok) {
                    f_stage<NTN, NQ, CHAIN>(ring + (size_t)sa * kFStage, ((4 * t) & 7) * 2, 4 * t, kp * NQ, txh, rt,
                                            lane, y, yb);
                    f_stage<NTN, NQ, CHAIN>(ring + (size_t)sb * kFStage, ((4 * t + 4) & 7) * 2, 4 * t + 4, kp * NQ, txh,
                                            rt, lane, y, yb);
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {  // the stages' data is consumed before release
                        hold_regs(y[j]);
                        hold_regs(yb[j]);
                    }
                }
                __syncwarp();
                if (wok && lane == 0) {
                    mbar_arrive(&empty[sa]);
                    mbar_arrive(&empty[sb]);
                }
            }
            {
                const int r0 = kp * kFRows + 16 * rt + g;
#pragma unroll
                for (int j = 0; j < NTN; ++j) {
                    const float2 cv = fold_weights<CHAIN>(cs, j, tq);
                    const float2 pp = i8_combine(y[j], yb[j], cv, tq);
                    const int m = 2 * j + (tq >> 1);
                    const float rfm = __shfl_sync(0xffffffffu, rfl, m & 31);
                    if ((tq & 1) == 0 && m < M) {
                        out[r0 * MS + m] = pp.x * rfm;
                        out[(r0 + 8) * MS + m] = pp.y * rfm;
                    }
                }
            }
            FUSED_MARK(L, 2);
            if (cons_bar_or<W>(*abort != 0)) break;

            // ---- SwiGLU -> activation planes, copied into every CTA of the cluster ----------------------
            // one activation per thread (feature f of row m); the group's exponent and sum come from
            // the two warps of the row (shuffles, then a consumer barrier); the planes are written
            // byte by byte into this CTA's slot, which then goes to the seven peers as one bulk copy
            uint8_t* aqp = aq + (size_t)par * aq_bytes;
            uint8_t* slot_p = aqp + crank * SB;
            float* sxs = reinterpret_cast<float*>(slot_p + ncols * 64);
            float* sxe = sxs + ncols;
            float av[(64 * MS + W * 32 - 1) / (W * 32)];
            constexpr int NA = (64 * MS + W * 32 - 1) / (W * 32);  // activations per thread
#pragma unroll
            for (int i = 0; i < NA; ++i) {
                const int idx = tid + i * W * 32, m = idx >> 6, f = idx & 63;
                av[i] = 0.f;
                if (m < M) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int k = 0; k < KP; ++k) {
                        gv += out[(k * kFRows + f) * MS + m];
                        uv += out[(k * kFRows + 64 + f) * MS + m];
                    }
                    const float sg = 1.0f / (1.0f + expf(-gv));
                    av[i] = (sg * gv) * uv;
                }
                if ((idx >> 6) < MS) {  // warp-uniform: whole warps of rows below MS
                    const unsigned bm = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(av[i])));
                    float sm = av[i];
#pragma unroll
                    for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
                    if (lane == 0) {
                        xch[((f >> 5) * 4 + 0) * MS + m] = __uint_as_float(bm);
                        xch[((f >> 5) * 4 + 1) * MS + m] = sm;
                    }
                }
            }
            FUSED_MARK(L, 11);
            cons_bar<W>();
#pragma unroll
            for (int i = 0; i < NA; ++i) {
                const int idx = tid + i * W * 32, m = idx >> 6, f = idx & 63;
                if (m < M) {
                    const float gmax = fmaxf(xch[(0 * 4 + 0) * MS + m], xch[(1 * 4 + 0) * MS + m]);
                    const int e = row_exp(__float_as_uint(gmax));
                    const float qa = rintf(__fmul_rn(av[i], pow2f(13 - e)));
                    const int A = (int)qa;
                    const int B = __float2int_rn(__fmul_rn(fmaf(-qa, pow2f(e - 13), av[i]), pow2f(27 - e)));
                    const int i0 = (A + 64) >> 7, i2 = (B + 64) >> 7;
                    const int d[4] = {i0, A - (i0 << 7), i2, B - (i2 << 7)};
                    const int pos = plane_pos(f);
#pragma unroll
                    for (int p = 0; p < 4; ++p) slot_p[(4 * m + p) * 64 + pos] = (uint8_t)(d[p] & 0xff);
                    if (f == 0) {
                        sxs[4 * m] = __fmul_rn(xch[(0 * 4 + 1) * MS + m] + xch[(1 * 4 + 1) * MS + m], 64.0f);
                        sxe[4 * m] = pow2f(e);
                    }
                }
            }
            fence_proxy_async_smem();  // the slot is read by the bulk copies below
            cons_bar<W>();
            FUSED_MARK(L, 14);
            if (warp == 0 && lane < kFCluster) {
                const uint32_t ls = smem_u32(slot_p), lbar = smem_u32(&actbar[par]);
                if (lane > 0) {
                    const uint32_t dst = (crank + (uint32_t)lane) % kFCluster;
                    bulk_s2cluster(mapa_u32(ls, dst), ls, SB, mapa_u32(lbar, dst));
                } else {
                    mbar_arrive_expect_tx(&actbar[par], (kFCluster - 1) * SB);
                }
            } else if (L > 0 && tid >= 64) {
                // clear this CTA's slice of acc_{L+2} (complete words of acc_L show that every CTA has read
                // acc_{L-1}, which it reuses); the fence orders the zeros before this CTA's own adds of
                // layer L, which any later adder to acc_{L+2} waits for
                if (zero_slice(a.acc + (size_t)((L + 2) % 3) * MH, MH, c, G, tid - 64, W * 32 - 64)) fence_acq_rel_gpu();
            }
            armed = L;
            FUSED_MARK(L, 3);
            if (L == 0 && tid == 0 && !*abort) grid_wait(a.sync, (unsigned)G, a.wait_cycles, abort);  // acc_1 cleared
            wok = warp_wait_cluster(&actbar[par], (uint32_t)((L >> 1) & 1), abort, a.sync + 1, a.wait_cycles);
            if (cons_bar_or<W>(!wok || *abort != 0)) break;
            armed = -1;
            FUSED_MARK(L, 4);

            // ---- down_proj rows of this CTA x the cluster's 512 features -> counted fixed point ---------
            const FOperand txa{aqp, reinterpret_cast<const float*>(aqp + ncols * 64),
                               reinterpret_cast<const float*>(aqp + ncols * 64) + ncols, (int)SB, (int)(SB / 4)};
            const bool rows_here = 16 * rt < RB;
            for (int h = 0; h < nhalf; ++h) {
#pragma unroll
                for (int j = 0; j < NTN; ++j) y[j][0] = y[j][1] = y[j][2] = y[j][3] = yb[j][0] = yb[j][1] = 0.f;
                {  // the half's two stages as a pair (see the gate/up loop)
                    const int sa = slot;
                    const uint32_t pa = fpar;
                    if (++slot == S) {
                        slot = 0;
                        fpar ^= 1u;
                    }
                    const int sb = slot;
                    const uint32_t pb = fpar;
                    if (++slot == S) {
                        slot = 0;
                        fpar ^= 1u;
                    }
                    FUSED_READY(L, mbar_test_wait(&full[sa], pa) && mbar_test_wait(&full[sb], pb));
                    if (wok) wok = warp_wait(&full[sa], pa, abort);
                    if (wok) wok = warp_wait(&full[sb], pb, abort);
                    if (h == 0) FUSED_MARK(L, 7);
                    if (h == nhalf - 1) FUSED_MARK(L, 9);
                    if (wok && rows_here) {
                        f_stage<NTN, NQ, CHAIN>(ring + (size_t)sa * kFStage, 0, 0, kp * NQ, txa, rt, lane, y, yb);
                        f_stage<NTN, NQ, CHAIN>(ring + (size_t)sb * kFStage, 8, 4, kp * NQ, txa, rt, lane, y, yb);
#pragma unroll
                        for (int j = 0; j < NTN; ++j) {
                            hold_regs(y[j]);
                            hold_regs(yb[j]);
                        }
                    }
                    __syncwarp();
                    if (wok && lane == 0) {
                        mbar_arrive(&empty[sa]);
                        mbar_arrive(&empty[sb]);
                    }
                }
                if (wok && rows_here) {
                    const int lr0 = h * RB + 16 * rt + g, lr1 = lr0 + 8;  // rows within this CTA's range
                    const bool add_res = cj == 0 && kp == 0;
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        const float2 cv = fold_weights<CHAIN>(cs, j, tq);
                        const float2 pp = i8_combine(y[j], yb[j], cv, tq);
                        const int m = 2 * j + (tq >> 1);
                        if ((tq & 1) == 0 && m < M) {
                            long long f0 = to_fix(pp.x), f1 = to_fix(pp.y);
                            if (add_res) {
                                f0 += to_fix(res[lr0 * MS + m]);
                                f1 += to_fix(res[lr1 * MS + m]);
                            }
                            red_add_u64(accN + (size_t)m * H + rd0 + lr0, fix_word(f0));
                            red_add_u64(accN + (size_t)m * H + rd0 + lr1, fix_word(f1));
                        }
                    }
                }
            }
            FUSED_MARK(L, 5);
            if (cons_bar_or<W>(!wok || *abort != 0)) break;
        }
    }
    // Exit.  After the first cluster barrier no CTA issues another copy; a CTA that left the layer loop
    // early (an abort) with its activation barrier armed then waits, bounded, for the copies its peers
    // issued into it to land, and the second barrier keeps every CTA until all have done so: no CTA
    // leaves while a peer's copy may still write into its shared memory.
    // A CTA that aborted without arming (it left before its SwiGLU) cannot tell whether a peer already
    // copied into it, so it lets about 100 us pass (a copy of one slot lands within microseconds),
    // and the second barrier holds the whole cluster meanwhile.  The normal path waits for nothing.
    cluster_sync_all();
    if (warp < W && armed >= 0) {
        uint64_t* bar = &actbar[armed & 1];
        const uint32_t ph = (uint32_t)((armed >> 1) & 1);
        const unsigned long long t0 = cycles_now();
        while (!mbar_try_wait_cluster(bar, ph) && cycles_now() - t0 < (1ull << 22)) {
        }
    } else if (tid == 0 && *abort) {
        const unsigned long long t0 = cycles_now();
        while (cycles_now() - t0 < 200000ull) {
        }
    }
    cluster_sync_all();
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
int fused_ntn(int64_t m) { return m <= 2 ? 1 : (m <= 4 ? 2 : 4); }
// Consumer warps: 8 (measured at one row: 16 warps, each taking two groups of a stage, 5 % slower)
#ifndef FUSED_W1
#define FUSED_W1 8
#endif
int fused_warps(int ntn) { return ntn == 1 ? FUSED_W1 : 8; }

uint32_t plan_fused(FusedArgs& a, int M, int H) {
    const int ntn = fused_ntn(M), ncols = 8 * ntn, MS = 2 * ntn, W = fused_warps(ntn);
    const int HG = H / kGroup, RD = H / kFCluster;
    auto al = [](uint32_t v, uint32_t x) { return (v + x - 1) / x * x; };
    for (int S = 12; S >= 3; --S) {
        uint32_t off = 0;
        a.off_bar = off;
        off += al((2u * S + 2u) * 8u, 128);
        a.off_misc = off;
        off += al(64u + (uint32_t)(W + 8) * MS * 4u, 128);
        a.off_hq = off;
        off += (uint32_t)HG * ncols * 64;
        a.off_hxs = off;
        off += al((uint32_t)HG * ncols * 4, 128);
        a.off_hxe = off;
        off += al((uint32_t)HG * ncols * 4, 128);
        a.off_cs = off;
        off += al((uint32_t)ncols * 4, 128);
        a.off_aq = off;
        off += al(2u * kFCluster * ncols * 72, 128);
        a.off_out = off;
        off += al((uint32_t)(W / 8) * kFRows * MS * 4, 128);
        a.off_res = off;
        off += al((uint32_t)RD * MS * 4, 128);
        off = al(off, 1024);
        a.off_ring = off;
        off += (uint32_t)S * kFStage + 1024;  // + the alignment of the dynamic shared-memory base
        if (off <= kFSmemLimit) {
            a.S = S;
            return off;
        }
    }
    return 0;
}

template <int NTN, int W>
cudaError_t fused_config(int grid, uint32_t smem, bool pdl, cudaStream_t stream, cudaLaunchConfig_t& cfg,
                         cudaLaunchAttribute (&attr)[2]) {
    cudaError_t e =
        cudaFuncSetAttribute(fused_layers_kernel<NTN, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(fused_threads(W));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = kFCluster;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaSuccess;
}

template <int NTN, int W>
cudaError_t fused_max_clusters(uint32_t smem, int* n) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    cudaError_t e = fused_config<NTN, W>(kFCluster, smem, false, nullptr, cfg, attr);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveClusters(n, fused_layers_kernel<NTN, W>, &cfg);
}

template <int NTN, int W>
cudaError_t fused_launch(const FusedArgs& a, int grid, uint32_t smem, bool pdl, cudaStream_t stream) {
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    const cudaError_t e = fused_config<NTN, W>(grid, smem, pdl, stream, cfg, attr);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernelEx(&cfg, fused_layers_kernel<NTN, W>, a);
}

// Whether `grid` CTAs in clusters of 8 can all be resident at once on the current device (the layer
// waits need every CTA running).  Cached per device and activation width: plan_fused fills shared
// memory to within one ring stage of the limit at every hidden size, one CTA per SM, so the count
// does not depend on the exact size.
bool fused_coresident(int ntn, int grid, uint32_t smem) {
    static std::mutex mu;
    static int cache[64][3];  // [device][ntn index]: 0 unknown, else max active clusters + 1
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    const int ti = ntn == 1 ? 0 : (ntn == 2 ? 1 : 2);
    std::lock_guard<std::mutex> lk(mu);
    if (!cache[dev][ti]) {
        int n = 0;
        const cudaError_t e = ntn == 1   ? fused_max_clusters<1, FUSED_W1>(smem, &n)
                              : ntn == 2 ? fused_max_clusters<2, 8>(smem, &n)
                                         : fused_max_clusters<4, 8>(smem, &n);
        if (e != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cache[dev][ti] = n + 1;
    }
    return (cache[dev][ti] - 1) * kFCluster >= grid;
}

}  // namespace

size_t fused_acc_bytes(int64_t m, int64_t hidden) { return (size_t)3 * (size_t)m * (size_t)hidden * 8; }

bool fused_supported(int64_t m, int64_t hidden, int64_t inter, int n_layers) {
    if (m < 1 || m > kFusedMaxRows || n_layers < 1 || n_layers > kFusedMaxLayers) return false;
    if (hidden != 512 && hidden != 1024 && hidden != 2048) return false;
    // inter / 64 CTAs on distinct SMs; the count field holds up to 31 contributions per word
    const int64_t G = inter / kGroup;
    if (inter % 512 != 0 || G > device_num_sms() || (fused_warps(fused_ntn(m)) / 8) * (G / kFCluster) > 31 ||
        tmap_encode_fn() == nullptr)
        return false;
    FusedArgs a;
    const uint32_t smem = plan_fused(a, (int)m, (int)hidden);
    return smem != 0 && fused_coresident(fused_ntn(m), (int)G, smem);
}

cudaError_t launch_fused_layers(const FusedLaunch& F, cudaStream_t stream) {
    static FusedArgs a;  // 28 KB: kept off the stack (the launch copies it)
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    a = FusedArgs{};
    const int M = (int)F.m, H = (int)F.hidden;
    const uint32_t smem = plan_fused(a, M, H);
    if (!smem) return cudaErrorInvalidConfiguration;
    const int RD = H / kFCluster, RB = std::min(RD, kFRows);
    for (int l = 0; l < F.n_layers; ++l) {
        const FusedLayer& Ly = F.layers[l];
        FusedLayerMaps& mp = a.lay[l];
        if (!encode_q4_maps(Ly.gate, 64, &mp.g, &mp.gs, &mp.gb) || !encode_q4_maps(Ly.up, 64, &mp.u, &mp.us, &mp.ub) ||
            !encode_q4_maps(Ly.down, RB, &mp.d, &mp.ds, &mp.db))
            return cudaErrorInvalidValue;
        a.norm_w[l] = Ly.norm_w;
    }
    a.h0 = F.h0;
    a.acc = F.acc;
    a.sync = F.sync;
    a.wait_cycles = F.wait_cycles;
    a.M = M;
    a.H = H;
    a.n_layers = F.n_layers;
    a.eps = F.eps;
    const int grid = (int)(F.inter / kGroup);
    switch (fused_ntn(M)) {
        case 1: return fused_launch<1, FUSED_W1>(a, grid, smem, F.pdl, stream);
        case 2: return fused_launch<2, 8>(a, grid, smem, F.pdl, stream);
        default: return fused_launch<4, 8>(a, grid, smem, F.pdl, stream);
    }
}

int fused_device_error(bool clear) { return tu_device_error(clear); }

}  // namespace marlin
