// q4_gemv.cu — Q4 (group-64 affine, MLX layout) decode GEMV / skinny GEMM for sm_100a.
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) on the decode path of
// marlin-mlx (src/model/marlin.cpp:18-25 qmatmul, :31-35 mlp_forward, :161-169 lm_head) and the
// greedy mx::argmax that follows the lm_head (src/sampling/sampler.cpp:14-16).
//
// Data path:
//   * Weights stream HBM -> shared memory by 1-D TMA bulk copies (cp.async.bulk; one per packed row
//     into a padded row so the fragment loads are bank-conflict free, one each for a block's scales
//     and biases).  The decode kernels issue them BEFORE griddepcontrol.wait: launched with
//     programmatic stream serialization, a kernel fetches its weights while its predecessor runs.
//   * Activations (optionally RMSNorm'ed on the fly) become bf16 planes — 1 for bf16 activations,
//     3 exact hi/mid/lo planes for binary32 — stored pre-permuted in mma.sync A-fragment order,
//     with per-(plane row, 64-group) sums.
//   * K is split across the warps of a CTA: each warp loads a group's A fragments once and reuses
//     them for all the CTA's 8-row weight tiles.  Nibbles become bf16 (1 + q/16) with one LOP3 per
//     pair (exact); mma.sync m16n8k16 (bf16 in, fp32 accumulate; weights as the B operand, 8 rows
//     per n8 tile) gives per group D = sum x*(1+q/16), folded as
//        y += 16*s*D + (b - 16*s)*sum(x)  ==  s*sum(x*q) + b*sum(x)
//     so the per-group scale/bias stay binary32 as in the reference's dequant formula.  Partials
//     meet in shared memory for the epilogue (store / SwiGLU of gate+up rows / residual add).
//
// Why mma.sync and not tcgen05 here: at M <= 32 the kernel is HBM-bound at 0.5625 B/weight; a
// tcgen05 operand must sit in shared memory in bf16, i.e. 2 B/weight written plus 2 B/weight read
// per weight, which exceeds shared-memory bandwidth at HBM rate.  Register-level dequant feeding
// mma.sync keeps the dequantized weights out of shared memory.
//
// The lm_head kernel is persistent: a producer warp streams 32-row vocabulary blocks through a
// TMA ring, 8 consumer warps split K, and the argmax is reduced on the fly with packed
// (ordered value << 32 | ~index) keys, one atomicMax per CTA and row, the last CTA decoding and
// re-zeroing the keys.  Logits are never written to memory.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_stage.cuh"
#include "q4_i8.cuh"

#include <cuda.h>

#include <algorithm>
#include <atomic>

namespace marlin {
namespace {

// ------------------------------------------------------------------------------------------------
// shared-memory geometry
// ------------------------------------------------------------------------------------------------
// Packed row stride in shared memory: K/2 bytes padded so the row stride in 4-byte words is 8 mod
// 32 (rows g = 0..3 of a half-warp then hit disjoint banks in the fragment loads).
__host__ __device__ inline int packed_row_stride(int K) {
    int words = K / 8;
    int pad = ((8 - (words % 32)) % 32 + 32) % 32;
    return (words + pad) * 4;
}
// bytes of one 8-row weight tile in shared memory: packed rows, scales [8][G], biases [8][G]
__host__ __device__ inline uint32_t tile_bytes(int K) {
    int G = K / kGroup;
    return align_up(8u * packed_row_stride(K) + 2u * 8u * G * 2u, 128);
}

// Whole-K staging.  When the activations fit in two 8-element units per thread: one pass (load,
// sums of squares, row factors, planes — one global round trip).  Otherwise norm factors in one
// pass and planes in a second (an L1 hit).  Ends with __syncthreads.
__device__ void stage_all(const void* x, int dtype, int K, const uint16_t* norm_w, float eps, const XGeom& g) {
    const int nt = blockDim.x;
    const int upr = K / 8, total = g.M * upr;
    if (total > 2 * nt) {
        if (norm_w) norm_factors_only(x, dtype, K, eps, g);
        stage_chunk(x, dtype, K, norm_w, 0, K / kGroup, g);
        return;
    }
    float v[2][8];
    uint4 nwv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int idx = (int)threadIdx.x + u * nt;
        if (idx < total) {
            const int k = (idx % upr) * 8;
            load8(x, dtype, (int64_t)(idx / upr) * K + k, v[u]);
            if (norm_w) nwv[u] = *reinterpret_cast<const uint4*>(norm_w + k);
        }
    }
    if (norm_w) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int idx = (int)threadIdx.x + u * nt;
            if (idx < total) g.ssq[idx] = unit_ssq(v[u], dtype);
        }
        __syncthreads();
        finish_norm_factors(dtype, g.M, K, eps, g);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int idx = (int)threadIdx.x + u * nt;  // idx % 32 == lane: groups are lane-aligned
        const bool ok = idx < total;
        emit_unit(v[u], nwv[u], ok ? idx / upr : 0, ok ? idx % upr : 0, ok, norm_w != nullptr, g);
    }
    __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// tensor-core group step
// ------------------------------------------------------------------------------------------------
template <int MT, bool HALF>
__device__ __forceinline__ void load_a(const uint8_t* xp, int XRS, const float* xs, int GC, int M_eff, int gl,
                                       uint32_t (&A)[MT][2][8], float (&X)[MT][2]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = mt * 16 + h * 8 + g;
            if ((HALF && h == 1) || r >= M_eff) {
#pragma unroll
                for (int j = 0; j < 8; ++j) A[mt][h][j] = 0u;
                X[mt][h] = 0.f;
            } else {
                const uint8_t* p = xp + (uint32_t)r * XRS + gl * 128 + t * 32;
                const uint4 lo = lds128(p), hi = lds128(p + 16);
                A[mt][h][0] = lo.x; A[mt][h][1] = lo.y; A[mt][h][2] = lo.z; A[mt][h][3] = lo.w;
                A[mt][h][4] = hi.x; A[mt][h][5] = hi.y; A[mt][h][6] = hi.z; A[mt][h][7] = hi.w;
                X[mt][h] = xs[r * GC + gl];
            }
        }
    }
}

// One 64-group of one 8-row tile: D = x . (1 + q/16) as two independent 2-step mma chains
// (steps 0-1 and 2-3), folded into acc with the group's (16 s, b - 16 s) for rows (2t, 2t+1).
template <int MT, bool HALF>
__device__ __forceinline__ void group_mma(const uint32_t (&A)[MT][2][8], const float (&X)[MT][2], uint2 wv,
                                          float4 sb, float (&acc)[MT][4]) {
    uint32_t p0[4], p1[4];
    q4_pairs(wv.x, p0);
    q4_pairs(wv.y, p1);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
        mma_bf16_16816(d0, A[mt][0][0], A[mt][1][0], A[mt][0][1], A[mt][1][1], p0[0], p0[1]);
        mma_bf16_16816(d1, A[mt][0][4], A[mt][1][4], A[mt][0][5], A[mt][1][5], p1[0], p1[1]);
        mma_bf16_16816(d0, A[mt][0][2], A[mt][1][2], A[mt][0][3], A[mt][1][3], p0[2], p0[3]);
        mma_bf16_16816(d1, A[mt][0][6], A[mt][1][6], A[mt][0][7], A[mt][1][7], p1[2], p1[3]);
        acc[mt][0] = fmaf(sb.x, d0[0] + d1[0], fmaf(sb.y, X[mt][0], acc[mt][0]));
        acc[mt][1] = fmaf(sb.z, d0[1] + d1[1], fmaf(sb.w, X[mt][0], acc[mt][1]));
        if (!HALF) {
            acc[mt][2] = fmaf(sb.x, d0[2] + d1[2], fmaf(sb.y, X[mt][1], acc[mt][2]));
            acc[mt][3] = fmaf(sb.z, d0[3] + d1[3], fmaf(sb.w, X[mt][1], acc[mt][3]));
        }
    }
}

// Scale-table entry of one (row, group): (16*s, b - 16*s).
__device__ __forceinline__ float2 sb_entry(float s, float b) {
    const float s16 = s * 16.0f;
    return make_float2(s16, b - s16);
}

// ------------------------------------------------------------------------------------------------
// TMA issue helpers
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ int64_t rows_in(const Q4Mat& W, int64_t row0, int64_t R) {
    return (int64_t)min((long long)R, max((long long)0, (long long)(W.n - row0)));
}
// Bytes the copies of an R-row block (rows [row0, row0 + R) of W) deliver: packed rows always,
// scales/biases only for a full block (a partial block's are read with plain loads).
__device__ __forceinline__ uint32_t block_bytes(const Q4Mat& W, int64_t row0, int R) {
    const int64_t rows = rows_in(W, row0, R);
    const int G = (int)(W.k / kGroup);
    uint32_t bytes = (uint32_t)(rows * (W.k / 2));
    if (rows == R) bytes += 2u * (uint32_t)R * G * 2u;
    return bytes;
}
// Copies into: packed rows at dst + r*RS, scales at sdst [R][G], biases at sdst + R*G*2 bytes.
__device__ __forceinline__ void issue_block(const Q4Mat& W, int64_t row0, int R, uint8_t* dst, int RS,
                                            uint8_t* sdst, uint64_t* bar) {
    const int64_t rows = rows_in(W, row0, R);
    const int G = (int)(W.k / kGroup);
    const uint32_t rb = (uint32_t)(W.k / 2);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(W.w) + row0 * (int64_t)rb;
    for (int r = 0; r < rows; ++r) tma_bulk_g2s(dst + r * RS, src + (int64_t)r * rb, rb, bar);
    if (rows == R) {
        tma_bulk_g2s(sdst, W.s + row0 * G, (uint32_t)R * G * 2u, bar);
        tma_bulk_g2s(sdst + R * G * 2, W.b + row0 * G, (uint32_t)R * G * 2u, bar);
    }
}

// ------------------------------------------------------------------------------------------------
// weight block layouts in shared memory
// ------------------------------------------------------------------------------------------------
// Row copies (any K): each packed row is one 1-D bulk copy into a row padded to RS bytes; tile
// column n of the mma is physical row n.  Used when a block has fewer than 32 rows (boxes would be
// under 4 KB) — with K >= 4096 the rows are >= 2 KB, which keeps the copy engine efficient.
//
// Swizzled boxes (2-D tensor map, 128-byte swizzle): a block of BR rows arrives as ceil(K/256)
// boxes of [BR rows x 128 B] (4 KB at BR = 32), box c holding words [32c, 32c+32) of every row; the
// hardware XORs the 16-byte unit index of row r with r & 7.  Tile column n maps to physical row
// perm(n) = 2(n&3) + (n>>2), so a half-warp's four rows are {0,2,4,6} (or {1,3,5,7}) and the
// XORed units of one 64-group are all distinct: conflict-free 8-byte fragment loads.
__device__ __forceinline__ int col_to_row(int n) { return 2 * (n & 3) + (n >> 2); }

// Address of the 8 packed bytes thread (g, t4) feeds the mma for tile row block `r8` (multiple of
// 8), group gg.
template <bool SWZ>
__device__ __forceinline__ const uint8_t* frag_addr(const uint8_t* blk, int BR, int RS, int r8, int g, int t4, int gg) {
    if (SWZ) {
        const int pr = col_to_row(g);
        const int j = (2 * (gg & 3) + (t4 >> 1)) ^ pr;
        return blk + (gg >> 2) * (BR * 128) + (r8 + pr) * 128 + j * 16 + (t4 & 1) * 8;
    }
    return blk + (r8 + g) * RS + gg * 32 + t4 * 8;
}

// ------------------------------------------------------------------------------------------------
// decode GEMV (one CTA per row block, weights fetched before the PDL wait)
// ------------------------------------------------------------------------------------------------
// A CTA owns NT 8-row tiles (kEpiSwiglu: NT/2 gate tiles and the NT/2 up tiles of the same
// features) and splits K over its NWK warps: the CTA stages the activations, then every warp runs
// its K range over all NT tiles, loading each group's A fragments once.
struct UnitArgs {
    CUtensorMap tm0, tm1;  // SWZ layout: tensor maps of w0 / w1 packed words [n][k/8]
    GemvLaunch L;
    int P, M_eff, G, NWK, GC, RS, XRS, BR, nchunk;
    uint32_t tbytes, off_tiles, off_sb, off_xp, off_xs, off_red, off_scr, off_bar;
};

__device__ __forceinline__ float swiglu_apply(float gv, float uv, int dtype) {
    if (dtype == kBF16) {
        const float gq = bf16_round(gv), uq = bf16_round(uv);
        const float sg = bf16_round(__fdividef(1.0f, 1.0f + expf(-gq)));
        const float tt = bf16_round(sg * gq);
        return bf16_round(tt * uq);
    }
    const float sg = 1.0f / (1.0f + expf(-gv));
    return (sg * gv) * uv;
}

template <int NT, int MT, bool HALF, int EPI, bool SWZ>
__global__ void __launch_bounds__(256, 2) q4_unit_kernel(const __grid_constant__ UnitArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const GemvLaunch& L = a.L;
    const int tid = threadIdx.x, wk = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int NWK = a.NWK, G = a.G;
    constexpr int HT = EPI == kEpiSwiglu ? NT / 2 : NT;  // output tiles (= tiles per matrix)
    constexpr int NMAT = EPI == kEpiSwiglu ? 2 : 1;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint8_t* wbase = smem + a.off_tiles;
    float2* sbt = reinterpret_cast<float2*>(smem + a.off_sb);  // [NT][G][8 columns]
    float* red = reinterpret_cast<float*>(smem + a.off_red);   // [NWK][NT][M_eff][8 columns]
    XGeom xg{smem + a.off_xp, reinterpret_cast<float*>(smem + a.off_xs),
             reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
             (int)L.m, a.P, a.M_eff, a.XRS, a.GC};

    const int64_t base = (int64_t)blockIdx.x * HT * 8;
    auto mat_of = [&](int t) -> int { return (EPI == kEpiSwiglu && t >= HT) ? 1 : 0; };
    auto tile_mat = [&](int t) -> const Q4Mat& { return mat_of(t) ? L.w1 : L.w0; };
    auto tile_row0 = [&](int t) -> int64_t { return base + (int64_t)(t % HT) * 8; };
    // SWZ: one block per matrix (packed boxes, then scales [BR][G], biases [BR][G]);
    // row copies: one tile per t (packed rows, scales [8][G], biases [8][G]).
    auto blk_of = [&](int t) -> uint8_t* { return SWZ ? wbase + mat_of(t) * a.tbytes : wbase + t * a.tbytes; };
    const int BR = SWZ ? a.BR : 8;
    const uint32_t packed = SWZ ? (uint32_t)a.nchunk * a.BR * 128 : 8u * a.RS;

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        uint32_t bytes = 0;
        if (SWZ) {
            for (int m = 0; m < NMAT; ++m) {
                bytes += packed;
                if (rows_in(m ? L.w1 : L.w0, base, BR) == BR) bytes += 2u * BR * G * 2u;
            }
            mbar_arrive_expect_tx(bar, bytes);
            for (int m = 0; m < NMAT; ++m) {
                const Q4Mat& W = m ? L.w1 : L.w0;
                const CUtensorMap* tm = m ? &a.tm1 : &a.tm0;
                uint8_t* blk = wbase + m * a.tbytes;
                for (int c = 0; c < a.nchunk; ++c) tma_load_2d(blk + c * BR * 128, tm, c * 32, (int32_t)base, bar);
                if (rows_in(W, base, BR) == BR) {
                    tma_bulk_g2s(blk + packed, W.s + base * G, (uint32_t)BR * G * 2u, bar);
                    tma_bulk_g2s(blk + packed + BR * G * 2, W.b + base * G, (uint32_t)BR * G * 2u, bar);
                }
            }
        } else {
#pragma unroll
            for (int t = 0; t < NT; ++t) bytes += block_bytes(tile_mat(t), tile_row0(t), 8);
            mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                uint8_t* tb = wbase + t * a.tbytes;
                issue_block(tile_mat(t), tile_row0(t), 8, tb, a.RS, tb + packed, bar);
            }
        }
    }
    // Everything above is independent of the previous kernel; activations below are not.
    pdl_wait();
    pdl_launch_dependents();

    const int K = (int)L.w0.k;
    const int g0 = wk * G / NWK, g1 = (wk + 1) * G / NWK;
    float acc[NT][MT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[t][mt][j] = 0.f;

    const bool chunked = a.GC < G;
    if (!chunked) stage_all(L.x, L.x_dtype, K, L.norm_w, L.eps, xg);
    else if (L.norm_w) norm_factors_only(L.x, L.x_dtype, K, L.eps, xg);

    // weights: uniform across the CTA — a (recorded) timeout ends the whole CTA
    if (!__syncthreads_and(mbar_wait(bar, 0) ? 1 : 0)) return;
    // scale table for this warp's groups of every tile, indexed by mma column
    // (partial blocks read their scales from global)
    {
        const int ng = g1 - g0, cnt = ng * 8 * NT;
        for (int e = lane; e < cnt; e += 32) {
            const int t = e / (ng * 8), rem = e - t * ng * 8, gg = g0 + (rem >> 3), n = rem & 7;
            const Q4Mat& W = tile_mat(t);
            const int pr = SWZ ? 8 * (t % HT) + col_to_row(n) : n;  // row within the smem block
            const int64_t row = (SWZ ? base : tile_row0(t)) + pr;
            float s = 0.f, b = 0.f;
            if (rows_in(W, SWZ ? base : tile_row0(t), BR) == BR) {
                const uint16_t* sp = reinterpret_cast<const uint16_t*>(blk_of(t) + packed);
                s = bf16_bits_to_f32(sp[pr * G + gg]);
                b = bf16_bits_to_f32(sp[BR * G + pr * G + gg]);
            } else if (row < W.n) {
                s = bf16_bits_to_f32(W.s[row * G + gg]);
                b = bf16_bits_to_f32(W.b[row * G + gg]);
            }
            sbt[(t * G + gg) * 8 + n] = sb_entry(s, b);
        }
    }
    __syncwarp();

    for (int gc0 = 0; gc0 < G; gc0 += a.GC) {
        const int ngc = min(a.GC, G - gc0);
        if (chunked) stage_chunk(L.x, L.x_dtype, K, L.norm_w, gc0, ngc, xg);
        const int lo = max(g0, gc0), hi = min(g1, gc0 + ngc);
#pragma unroll 1
        for (int gg = lo; gg < hi; ++gg) {
            uint32_t A[MT][2][8];
            float X[MT][2];
            load_a<MT, HALF>(xg.xp, a.XRS, xg.xs, a.GC, a.M_eff, gg - gc0, A, X);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint2 wv = lds64(frag_addr<SWZ>(blk_of(t), BR, a.RS, SWZ ? 8 * (t % HT) : 0, g, t4, gg));
                const float4 sb = *reinterpret_cast<const float4*>(sbt + (t * G + gg) * 8 + 2 * t4);
                group_mma<MT, HALF>(A, X, wv, sb, acc[t]);
            }
        }
        if (chunked) __syncthreads();  // chunk buffer reuse
    }

    // partials -> red[((wk*NT + t)*M_eff + r)*8 + column]
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < (HALF ? 1 : 2); ++h) {
                const int r = mt * 16 + h * 8 + g;
                if (r < a.M_eff)
                    *reinterpret_cast<float2*>(red + ((size_t)(wk * NT + t) * a.M_eff + r) * 8 + 2 * t4) =
                        make_float2(acc[t][mt][2 * h], acc[t][mt][2 * h + 1]);
            }
    __syncthreads();

    const int M = (int)L.m, P = a.P;
    auto gather = [&](int t, int m, int n) -> float {
        float v = 0.f;
        for (int w = 0; w < NWK; ++w)
            for (int p = 0; p < P; ++p) v += red[((size_t)(w * NT + t) * a.M_eff + (p * M + m)) * 8 + n];
        return v;
    };
    const int total = HT * M * 8;
    for (int o = tid; o < total; o += blockDim.x) {
        const int n = o & 7, rest = o >> 3, m = rest % M, t = rest / M;
        const int64_t row = tile_row0(t) + (SWZ ? col_to_row(n) : n);
        if (row >= L.w0.n) continue;
        const int64_t yi = (int64_t)m * L.ldy + row;
        float v;
        if (EPI == kEpiSwiglu) {
            v = swiglu_apply(gather(t, m, n), gather(t + HT, m, n), L.y_dtype);
        } else {
            v = gather(t, m, n);
            if (EPI == kEpiResid) v = load_act(L.resid, L.resid_dtype, (int64_t)m * L.ldr + row) + v;
        }
        if (L.y_dtype == kBF16)
            static_cast<uint16_t*>(L.y)[yi] = (uint16_t)f32_to_bf16_bits(v);
        else
            static_cast<float*>(L.y)[yi] = v;
    }
}

// ------------------------------------------------------------------------------------------------
// lm_head + argmax: persistent CTAs, producer warp + 8 consumer warps, 32-row blocks
// ------------------------------------------------------------------------------------------------
constexpr int kLmRows = 32;      // rows per block (4 tiles): 4 KB boxes
constexpr int kLmTiles = 4;
constexpr int kLmConsumers = 8;  // consumer warps (split K)
constexpr int kLmThreads = 32 * (kLmConsumers + 1);
constexpr int kLmMaxGroupsPerWarp = 8;

struct LmArgs {
    CUtensorMap tm;  // packed words [n][k/8], box [32 words][32 rows], 128-byte swizzle
    LmHeadLaunch L;
    int P, M_eff, G, XRS, S, nchunk;
    int64_t nblocks;
    uint32_t sbytes, packed, off_ring, off_sb, off_xp, off_xs, off_scr, off_bar, off_red, off_keys;
};

__device__ __forceinline__ unsigned long long pack_key(float v, int64_t idx) {
    uint32_t u = __float_as_uint(v);
    uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ void unpack_key(unsigned long long k, int32_t* id, float* v) {
    uint32_t o = (uint32_t)(k >> 32);
    uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    *v = __uint_as_float(u);
    *id = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
}

// Barrier among the 8 consumer warps (named barrier 1); returns the AND of `pred` over them.
__device__ __forceinline__ bool consumers_and(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(32 * kLmConsumers)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void lm_issue(const LmArgs& a, int64_t blk, uint8_t* st, uint64_t* bar) {
    const int64_t row0 = blk * kLmRows;
    const bool fullblk = rows_in(a.L.w, row0, kLmRows) == kLmRows;
    const int G = a.G;
    mbar_arrive_expect_tx(bar, a.packed + (fullblk ? 2u * kLmRows * G * 2u : 0u));
    for (int c = 0; c < a.nchunk; ++c) tma_load_2d(st + c * kLmRows * 128, &a.tm, c * 32, (int32_t)row0, bar);
    if (fullblk) {
        tma_bulk_g2s(st + a.packed, a.L.w.s + row0 * G, (uint32_t)kLmRows * G * 2u, bar);
        tma_bulk_g2s(st + a.packed + kLmRows * G * 2, a.L.w.b + row0 * G, (uint32_t)kLmRows * G * 2u, bar);
    }
}

template <int MT, bool HALF>
__global__ void __launch_bounds__(kLmThreads, 1) q4_lm_head_kernel(const __grid_constant__ LmArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const LmHeadLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int G = a.G, S = a.S;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* empty = full + S;
    uint8_t* ring = smem + a.off_ring;
    float* red = reinterpret_cast<float*>(smem + a.off_red);  // [2][8][M_eff][32 columns]
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(smem + a.off_keys);
    XGeom xg{smem + a.off_xp, reinterpret_cast<float*>(smem + a.off_xs),
             reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
             (int)L.m, a.P, a.M_eff, a.XRS, G};
    const bool producer = warp == kLmConsumers;

    if (tid == 0) {
        prefetch_tmap(&a.tm);
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kLmConsumers);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (producer && lane == 0) {
        for (int s = 0; s < S; ++s) {
            const int64_t blk = blockIdx.x + (int64_t)s * gridDim.x;
            if (blk >= a.nblocks) break;
            lm_issue(a, blk, ring + (size_t)s * a.sbytes, &full[s]);
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    stage_all(L.x, L.x_dtype, (int)L.w.k, L.norm_w, L.eps, xg);

    const int M = (int)L.m, P = a.P;
    constexpr int kSlots = 4;  // a lane owns rows m = (lane >> 2) + 8j, j < 4 (M <= 32)
    unsigned long long best[kSlots];
#pragma unroll
    for (int j = 0; j < kSlots; ++j) best[j] = 0ull;

    if (producer) {
        if (lane == 0) {
            for (int64_t i = S;; ++i) {
                const int64_t blk = blockIdx.x + i * gridDim.x;
                if (blk >= a.nblocks) break;
                const int s = (int)(i % S);
                if (!mbar_wait(&empty[s], (uint32_t)(((i / S) - 1) & 1))) break;
                lm_issue(a, blk, ring + (size_t)s * a.sbytes, &full[s]);
            }
        }
    } else {
        const int wk = warp;
        const int g0 = wk * G / kLmConsumers, g1 = (wk + 1) * G / kLmConsumers, ng = g1 - g0;
        float2* table = reinterpret_cast<float2*>(smem + a.off_sb) + (size_t)wk * kLmMaxGroupsPerWarp * kLmRows;
        for (int64_t i = 0;; ++i) {
            const int64_t blk = blockIdx.x + i * gridDim.x;
            if (blk >= a.nblocks) break;
            const int s = (int)(i % S);
            const uint8_t* st = ring + (size_t)s * a.sbytes;
            // uniform over the consumers: on a (recorded) timeout all of them stop together
            if (!consumers_and(mbar_wait(&full[s], (uint32_t)((i / S) & 1)))) break;
            const int64_t row0 = blk * kLmRows;
            const bool fullblk = rows_in(L.w, row0, kLmRows) == kLmRows;
            const uint16_t* sp = reinterpret_cast<const uint16_t*>(st + a.packed);
            // table[gl][column c]: the (16 s, b - 16 s) of physical row (c & ~7) + perm(c & 7)
            for (int e = lane; e < kLmMaxGroupsPerWarp * kLmRows; e += 32) {
                const int c = (e >> 2) & (kLmRows - 1), gl = (e & 3) + (e >> 7) * 4;
                if (gl >= ng) continue;
                const int gg = g0 + gl;
                const int pr = (c & ~7) + col_to_row(c & 7);
                float s_ = 0.f, b_ = 0.f;
                if (fullblk) {
                    s_ = bf16_bits_to_f32(sp[pr * G + gg]);
                    b_ = bf16_bits_to_f32(sp[kLmRows * G + pr * G + gg]);
                } else if (row0 + pr < L.w.n) {
                    s_ = bf16_bits_to_f32(L.w.s[(row0 + pr) * G + gg]);
                    b_ = bf16_bits_to_f32(L.w.b[(row0 + pr) * G + gg]);
                }
                table[gl * kLmRows + c] = sb_entry(s_, b_);
            }
            __syncwarp();
            float acc[kLmTiles][MT][4];
#pragma unroll
            for (int t = 0; t < kLmTiles; ++t)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[t][mt][j] = 0.f;
#pragma unroll 1
            for (int gl = 0; gl < ng; ++gl) {
                const int gg = g0 + gl;
                uint32_t A[MT][2][8];
                float X[MT][2];
                load_a<MT, HALF>(xg.xp, a.XRS, xg.xs, G, a.M_eff, gg, A, X);
#pragma unroll
                for (int t = 0; t < kLmTiles; ++t) {
                    const uint2 wv = lds64(frag_addr<true>(st, kLmRows, 0, t * 8, g, t4, gg));
                    const float4 sb = *reinterpret_cast<const float4*>(table + gl * kLmRows + t * 8 + 2 * t4);
                    group_mma<MT, HALF>(A, X, wv, sb, acc[t]);
                }
            }
#pragma unroll
            for (int t = 0; t < kLmTiles; ++t)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) hold_regs(acc[t][mt]);  // stage data consumed before release
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // this warp no longer reads stage s
            float* rb = red + (size_t)(i & 1) * kLmConsumers * a.M_eff * kLmRows;
#pragma unroll
            for (int t = 0; t < kLmTiles; ++t)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int h = 0; h < (HALF ? 1 : 2); ++h) {
                        const int r = mt * 16 + h * 8 + g;
                        if (r < a.M_eff)
                            *reinterpret_cast<float2*>(rb + ((size_t)wk * a.M_eff + r) * kLmRows + t * 8 + 2 * t4) =
                                make_float2(acc[t][mt][2 * h], acc[t][mt][2 * h + 1]);
                    }
            consumers_and(true);  // the block's partials are visible to all consumers
            // warp wk finishes columns [4wk, 4wk+4): lane -> column 4wk + (lane & 3), m = (lane >> 2) + 8j
            const int c = 4 * wk + (lane & 3);
            const int64_t row = row0 + (c & ~7) + col_to_row(c & 7);
            if (row < L.w.n) {
#pragma unroll
                for (int j = 0; j < kSlots; ++j) {
                    const int m = (lane >> 2) + 8 * j;
                    if (m < M) {
                        float v = 0.f;
                        for (int w = 0; w < kLmConsumers; ++w)
                            for (int p = 0; p < P; ++p) v += rb[((size_t)w * a.M_eff + p * M + m) * kLmRows + c];
                        if (L.x_dtype == kBF16 && !L.norm_w) v = bf16_round(v);
                        const unsigned long long k = pack_key(v, L.vocab_offset + row);
                        best[j] = k > best[j] ? k : best[j];
                    }
                }
            }
        }
        // reduce over the 4 lanes sharing m, then over warps
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
#pragma unroll
            for (int o = 1; o < 4; o <<= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[j], o);
                best[j] = other > best[j] ? other : best[j];
            }
        }
        if ((lane & 3) == 0) {
#pragma unroll
            for (int j = 0; j < kSlots; ++j) {
                const int m = (lane >> 2) + 8 * j;
                if (m < M) ckeys[wk * M + m] = best[j];
            }
        }
    }
    __syncthreads();
    __shared__ bool is_last;
    if (tid < M) {
        unsigned long long k = 0ull;
        for (int w = 0; w < kLmConsumers; ++w) k = ckeys[w * M + tid] > k ? ckeys[w * M + tid] : k;
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
            int32_t id;
            float v;
            unpack_key(k, &id, &v);
            if (L.ids) L.ids[tid] = id;
            if (L.best) L.best[tid] = v;
        }
        if (tid == 0) atomicExch(L.counter, 0u);
    }
}

__global__ void decode_keys_kernel(const unsigned long long* keys, int64_t m, int32_t* ids, float* best) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < m) {
        int32_t id;
        float v;
        unpack_key(keys[i], &id, &v);
        if (ids) ids[i] = id;
        if (best) best[i] = v;
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
int num_sms() { return device_sm_count(); }

constexpr uint32_t kSmemLimit = 225 * 1024;     // dynamic, incl. 1 KB alignment slack; leaves room for static
constexpr uint32_t kSmemTwoPerSm = 111 * 1024;  // two CTAs per SM (228 KB per SM, 1 KB reserved each)

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
    // looked up once; the initialisation of a function-local static is thread-safe
    static const EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<EncodeTiledFn>(p);
        return EncodeTiledFn(nullptr);
    }();
    return fn;
}

// Packed words of W as a 2-D tensor [n rows][k/8 words], box [32 words][box_rows rows], 128-byte
// swizzle, zero fill out of range.
bool encode_packed_map(CUtensorMap* m, const Q4Mat& W, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(W.k / 8), (cuuint64_t)W.n};
    const cuuint64_t strides[1] = {(cuuint64_t)(W.k / 2)};
    const cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(W.w), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename KernelT, typename ArgT>
cudaError_t launch_kernel(KernelT kernel, const ArgT& args, int grid, int threads, uint32_t smem, bool pdl,
                          cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

template <int NT, int EPI, bool SWZ>
cudaError_t dispatch_unit(const UnitArgs& a, int grid, int threads, uint32_t smem, bool pdl, cudaStream_t st) {
    if (a.M_eff <= 8) return launch_kernel(q4_unit_kernel<NT, 1, true, EPI, SWZ>, a, grid, threads, smem, pdl, st);
    if (a.M_eff <= 16) return launch_kernel(q4_unit_kernel<NT, 1, false, EPI, SWZ>, a, grid, threads, smem, pdl, st);
    return launch_kernel(q4_unit_kernel<NT, 2, false, EPI, SWZ>, a, grid, threads, smem, pdl, st);
}

// Shared-memory plan of the unit kernel; 0 if it does not fit.
uint32_t plan_unit(UnitArgs& a, int NT, int nmat, bool swz, int64_t M, bool norm, int K) {
    const int HT = NT / nmat;
    if (swz) {
        a.BR = HT * 8;
        a.nchunk = (K / 8 + 31) / 32;
        a.tbytes = align_up((uint32_t)a.nchunk * a.BR * 128 + 2u * a.BR * a.G * 2u, 1024);
    } else {
        a.BR = 8;
        a.nchunk = 0;
        a.tbytes = tile_bytes(K);
    }
    uint32_t off = 0;
    a.off_tiles = off;
    off += (swz ? nmat : NT) * a.tbytes;
    a.off_bar = off;
    off += 128;
    a.off_scr = off;
    off += align_up((64 + (norm ? (uint32_t)M * (K / 8) : 0u)) * 4, 128);
    a.off_sb = off;
    off += align_up((uint32_t)NT * a.G * 8 * 8, 128);
    a.off_red = off;
    off += align_up((uint32_t)a.NWK * NT * a.M_eff * 8 * 4, 128);
    const uint32_t fixed = off + 1024;  // + alignment slack of the dynamic window
    // whole-K activations when they fit under the two-CTAs-per-SM budget, else K chunks
    const uint32_t whole = align_up((uint32_t)a.M_eff * (a.G * 128 + 16), 128) + align_up((uint32_t)a.M_eff * a.G * 4, 128);
    int GC = a.G;
    if (fixed + whole > kSmemTwoPerSm) {
        const uint32_t budget = std::max<uint32_t>(kSmemTwoPerSm, fixed + 16384);
        const uint32_t per_group = (uint32_t)a.M_eff * (128 + 4);
        GC = (int)((budget - fixed - (uint32_t)a.M_eff * 16 - 256) / per_group);
        GC = std::max(1, std::min(GC, a.G));
    }
    a.GC = GC;
    a.XRS = GC * 128 + 16;
    a.off_xp = off;
    off += align_up((uint32_t)a.M_eff * a.XRS, 128);
    a.off_xs = off;
    off += align_up((uint32_t)a.M_eff * GC * 4, 128);
    off += 1024;  // alignment slack
    return off <= kSmemLimit ? off : 0;
}

}  // namespace

std::atomic<int> g_decode_path{kPathI8};  // process-wide, set from any thread

int decode_path() { return g_decode_path; }

bool set_decode_path(int path) {
    if (path != kPathI8 && path != kPathBf16) return false;
    g_decode_path = path;
    return true;
}

int gemv_max_rows(int act_dtype, bool normed, int64_t k) {
    if (path_is_i8(g_decode_path) && i8_supported(k, 1)) return kI8MaxRows;
    return (normed || act_dtype == kF32) ? 10 : 32;
}
int lm_head_max_rows(int act_dtype, bool normed, int64_t k) {
    if (path_is_i8(g_decode_path) && i8_supported(k, 1)) return kI8MaxRows;
    const bool p3 = normed || act_dtype == kF32;
    return p3 ? 5 : 16;
}

cudaError_t launch_q4_gemv(const GemvLaunch& L, cudaStream_t stream) {
    if (path_is_i8(g_decode_path) && i8_supported(L.w0.k, L.m)) return launch_i8_gemv(L, stream);
    UnitArgs a{};
    a.L = L;
    const int K = (int)L.w0.k;
    a.G = K / kGroup;
    a.P = (L.norm_w || L.x_dtype == kF32) ? 3 : 1;
    a.M_eff = (int)L.m * a.P;
    a.RS = packed_row_stride(K);
    a.NWK = std::max(1, std::min(8, a.G / 4));
    const int epi = L.epi;
    const int nmat = epi == kEpiSwiglu ? 2 : 1;
    const int64_t want = (int64_t)num_sms() * 5 / 4;  // CTAs wanted: about one wave
    // tiles per CTA: as many as keep >= ~1.25 CTAs per SM
    int NT = nmat;
    for (int c : {8, 4, 2}) {
        if (c < nmat || (epi != kEpiSwiglu && c > 4)) continue;
        const int64_t ctas = (L.w0.n + (c / nmat) * 8 - 1) / ((c / nmat) * 8);
        if (ctas >= want && (a.M_eff <= 8 || c <= 4)) {
            NT = c;
            break;
        }
    }
    uint32_t smem = 0;
    bool swz = false;
    for (; NT >= nmat; NT /= 2) {
        swz = (NT / nmat) * 8 >= 32 && encode_fn() != nullptr;
        smem = plan_unit(a, NT, nmat, swz, L.m, L.norm_w != nullptr, K);
        if (smem) break;
    }
    if (!smem) return cudaErrorInvalidConfiguration;
    if (swz) {
        if (!encode_packed_map(&a.tm0, L.w0, a.BR)) return cudaErrorInvalidValue;
        if (nmat == 2 && !encode_packed_map(&a.tm1, L.w1, a.BR)) return cudaErrorInvalidValue;
    }
    const int64_t rows_per_cta = (NT / nmat) * 8;
    const int grid = (int)((L.w0.n + rows_per_cta - 1) / rows_per_cta);
    if (grid <= 0) return cudaSuccess;
    const int threads = 32 * a.NWK;
    if (epi == kEpiSwiglu) {
        if (NT == 8) return dispatch_unit<8, kEpiSwiglu, true>(a, grid, threads, smem, L.pdl, stream);
        if (NT == 4) return swz ? dispatch_unit<4, kEpiSwiglu, true>(a, grid, threads, smem, L.pdl, stream)
                                : dispatch_unit<4, kEpiSwiglu, false>(a, grid, threads, smem, L.pdl, stream);
        return dispatch_unit<2, kEpiSwiglu, false>(a, grid, threads, smem, L.pdl, stream);
    }
    if (epi == kEpiResid) {
        if (NT == 4) return swz ? dispatch_unit<4, kEpiResid, true>(a, grid, threads, smem, L.pdl, stream)
                                : dispatch_unit<4, kEpiResid, false>(a, grid, threads, smem, L.pdl, stream);
        if (NT == 2) return dispatch_unit<2, kEpiResid, false>(a, grid, threads, smem, L.pdl, stream);
        return dispatch_unit<1, kEpiResid, false>(a, grid, threads, smem, L.pdl, stream);
    }
    if (NT == 4) return swz ? dispatch_unit<4, kEpiStore, true>(a, grid, threads, smem, L.pdl, stream)
                            : dispatch_unit<4, kEpiStore, false>(a, grid, threads, smem, L.pdl, stream);
    if (NT == 2) return dispatch_unit<2, kEpiStore, false>(a, grid, threads, smem, L.pdl, stream);
    return dispatch_unit<1, kEpiStore, false>(a, grid, threads, smem, L.pdl, stream);
}

cudaError_t launch_q4_lm_head_argmax(const LmHeadLaunch& L, cudaStream_t stream) {
    if (path_is_i8(g_decode_path) && i8_supported(L.w.k, L.m)) return launch_i8_lm_head(L, stream);
    LmArgs a{};
    a.L = L;
    const int K = (int)L.w.k;
    a.G = K / kGroup;
    if (a.G > kLmMaxGroupsPerWarp * kLmConsumers) return cudaErrorInvalidValue;
    a.P = (L.norm_w || L.x_dtype == kF32) ? 3 : 1;
    a.M_eff = (int)L.m * a.P;
    if (a.M_eff > 32 || L.m > 32) return cudaErrorInvalidValue;
    if (!encode_packed_map(&a.tm, L.w, kLmRows)) return cudaErrorInvalidValue;
    a.nchunk = (K / 8 + 31) / 32;
    a.XRS = a.G * 128 + 16;
    a.nblocks = (L.w.n + kLmRows - 1) / kLmRows;
    a.packed = (uint32_t)a.nchunk * kLmRows * 128;
    a.sbytes = align_up(a.packed + 2u * kLmRows * a.G * 2u, 1024);
    uint32_t off = 0;
    a.off_bar = off;
    off += 256;
    a.off_scr = off;
    off += align_up((64 + (L.norm_w ? (uint32_t)L.m * (K / 8) : 0u)) * 4, 128);
    a.off_keys = off;
    off += align_up(kLmConsumers * (uint32_t)L.m * 8, 128);
    a.off_red = off;
    off += align_up(2u * kLmConsumers * a.M_eff * kLmRows * 4, 128);
    a.off_sb = off;
    off += align_up((uint32_t)kLmConsumers * kLmMaxGroupsPerWarp * kLmRows * 8, 128);
    a.off_xp = off;
    off += align_up((uint32_t)a.M_eff * a.XRS, 128);
    a.off_xs = off;
    off += align_up((uint32_t)a.M_eff * a.G * 4, 128);
    off = align_up(off, 1024);  // 128-byte-swizzled TMA boxes need 1024-byte-aligned destinations
    a.off_ring = off;
    const uint32_t avail = kSmemLimit > off + 1024 ? kSmemLimit - off - 1024 : 0;
    a.S = std::min<int>(12, (int)(avail / a.sbytes));  // 2*S mbarriers fit the 256-byte slot
    if (a.S < 2) return cudaErrorInvalidConfiguration;
    const uint32_t smem = off + (uint32_t)a.S * a.sbytes + 1024;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), a.nblocks));
    if (a.M_eff <= 8) return launch_kernel(q4_lm_head_kernel<1, true>, a, grid, kLmThreads, smem, L.pdl, stream);
    if (a.M_eff <= 16) return launch_kernel(q4_lm_head_kernel<1, false>, a, grid, kLmThreads, smem, L.pdl, stream);
    return launch_kernel(q4_lm_head_kernel<2, false>, a, grid, kLmThreads, smem, L.pdl, stream);
}

int gemv_device_error(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_marlin_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_marlin_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

cudaError_t launch_decode_keys(const unsigned long long* keys, int64_t m, int32_t* ids, float* best,
                               cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    decode_keys_kernel<<<(unsigned)((m + 127) / 128), 128, 0, stream>>>(keys, m, ids, best);
    return cudaGetLastError();
}

}  // namespace marlin
