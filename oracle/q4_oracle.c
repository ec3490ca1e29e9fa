/*
 * q4_oracle.c — CPU restatement of marlin-mlx's Q4 path.  TEST INFRASTRUCTURE ONLY: the checker
 * for the CUDA product, never linked into it.  PARITY UNPINNED (see q4_oracle.h): MLX v0.25.2,
 * which owns the arithmetic in the reference, is not present and the reference has no tests.
 *
 * Build: oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).  Every float operation below is a
 * single IEEE binary32 operation with round-to-nearest-even; sums use the fixed order written
 * next to them, so results are reproducible across thread counts.
 */
#include "q4_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int q4o_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- scalar helpers ------------------------------------------------------------------------- */
float q4o_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t q4o_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf16_round(float f) { return q4o_bf16_to_f32(q4o_f32_to_bf16(f)); }

static inline float load_x(const void* x, int dtype, int64_t i) {
    return dtype == Q4O_BF16 ? q4o_bf16_to_f32(((const uint16_t*)x)[i]) : ((const float*)x)[i];
}

/* ---- generator ------------------------------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z) { /* splitmix64 finaliser */
    z ^= z >> 30;
    z *= 0xbf58476d1ce4e5b9ull;
    z ^= z >> 27;
    z *= 0x94d049bb133111ebull;
    z ^= z >> 31;
    return z;
}

uint16_t q4o_synth_bf16_at(uint64_t seed, uint64_t i, float mean, float sigma) {
    uint64_t base = mix64(seed ^ 0x5851f42d4c957f2dull);
    int64_t s = 0;
    for (uint64_t r = 0; r < 3; ++r) {
        uint64_t h = mix64(base + (3u * i + r) * 0x9e3779b97f4a7c15ull);
        s += (int64_t)((h & 0xffffu) + ((h >> 16) & 0xffffu) + ((h >> 32) & 0xffffu) + (h >> 48));
    }
    float z = (float)(s - 393210); /* exact: |s - 393210| <= 393210 < 2^24 */
    float v = z * (sigma * (1.0f / 65536.0f));
    v = v + mean;
    return q4o_f32_to_bf16(v);
}

void q4o_synth_bf16(uint16_t* out, int64_t n, uint64_t seed, float mean, float sigma) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = q4o_synth_bf16_at(seed, (uint64_t)i, mean, sigma);
}

/* ---- quantize --------------------------------------------------------------------------------
 * Restates MLX's affine quantization (mlx::core::quantize, v0.25.2) as called by the reference at
 * src/model/weights.cpp:46 (quantize_weight, :45-56) and :183 (lm_head).  Per row and per
 * contiguous group of 64 along K, in binary32:
 *   max = max(0, w...)  [Q4O_TRUE_MINMAX: max(w...)],   min = min(w...)
 *   s   = max((max - min) / 15, 1e-7)
 *   side = |min| > |max|;  s = side ? s : -s;  edge = side ? min : max
 *   q0  = round(edge / s);  if q0 != 0: s = edge / q0, b = edge  else b = 0     (zero snapping)
 *   q_j = clamp(round((w_j - b) / s), 0, 15)      (s, b in binary32 here; stored as bf16)
 * round = ties away from zero [Q4O_ROUND_HALF_EVEN: ties to even].  Packing: nibble j of word i
 * holds element 8i+j in bits [4j, 4j+4) (little-endian, low nibble first). */
static inline float q4o_round(float v, unsigned flags) {
    return (flags & Q4O_ROUND_HALF_EVEN) ? rintf(v) : roundf(v);
}

int q4o_quantize(const uint16_t* w, int64_t N, int64_t K, int group_size, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases, unsigned flags) {
    if (group_size != Q4O_GROUP || bits != Q4O_BITS || N < 0 || K <= 0 || K % Q4O_GROUP) return -1;
    const int64_t G = K / Q4O_GROUP;
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t g = 0; g < G; ++g) {
            const uint16_t* src = w + n * K + g * Q4O_GROUP;
            float vals[Q4O_GROUP];
            float wmin = INFINITY;
            float wmax = (flags & Q4O_TRUE_MINMAX) ? -INFINITY : 0.0f;
            for (int j = 0; j < Q4O_GROUP; ++j) {
                vals[j] = q4o_bf16_to_f32(src[j]);
                wmin = fminf(wmin, vals[j]);
                wmax = fmaxf(wmax, vals[j]);
            }
            float scale = fmaxf((wmax - wmin) / 15.0f, 1e-7f);
            float bias;
            if (flags & Q4O_NO_ZERO_SNAP) {
                bias = wmin;
            } else {
                int side = fabsf(wmin) > fabsf(wmax);
                scale = side ? scale : -scale;
                float edge = side ? wmin : wmax;
                float q0 = q4o_round(edge / scale, flags);
                if (q0 != 0.0f) {
                    scale = edge / q0;
                    bias = edge;
                } else {
                    bias = 0.0f;
                }
            }
            uint16_t s16 = q4o_f32_to_bf16(scale), b16 = q4o_f32_to_bf16(bias);
            if (flags & Q4O_BF16_PARAMS_FIRST) {
                scale = q4o_bf16_to_f32(s16);
                bias = q4o_bf16_to_f32(b16);
            }
            scales[n * G + g] = s16;
            biases[n * G + g] = b16;
            for (int i = 0; i < Q4O_GROUP / 8; ++i) {
                uint32_t word = 0;
                for (int j = 0; j < 8; ++j) {
                    float c = q4o_round((vals[8 * i + j] - bias) / scale, flags);
                    c = fminf(fmaxf(c, 0.0f), 15.0f);
                    word |= (uint32_t)c << (4 * j);
                }
                wq[n * (K / 8) + g * 8 + i] = word;
            }
        }
    }
    return 0;
}

float q4o_dequant_at(const q4o_tensor* t, int64_t n, int64_t k) {
    const int64_t G = t->K / Q4O_GROUP;
    uint32_t word = t->weight[n * (t->K / 8) + k / 8];
    float q = (float)((word >> (4 * (k % 8))) & 15u);
    float s = q4o_bf16_to_f32(t->scales[n * G + k / Q4O_GROUP]);
    float b = q4o_bf16_to_f32(t->biases[n * G + k / Q4O_GROUP]);
    return s * q + b;
}

/* ---- quantized matmul ------------------------------------------------------------------------
 * y[m,n] = sum_g ( s*acc + b*xs ) with acc = sum_{k in g} x*q, xs = sum_{k in g} x, the per-group
 * decomposition of scale*q+bias that MLX's quantized matmul uses.  Order: acc and xs are each eight
 * lanes (k mod 8, ascending k) reduced as ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)); then
 * t = s*acc + b*xs, y += t over ascending g. */
static inline float lanes_sum8(const float* l) {
    return ((l[0] + l[1]) + (l[2] + l[3])) + ((l[4] + l[5]) + (l[6] + l[7]));
}

int q4o_qmatmul(const void* x, int x_dtype, int64_t M, const q4o_tensor* w, float* y32) {
    const int64_t K = w->K, N = w->N;
    if (K <= 0 || K % Q4O_GROUP || M < 0 || N < 0) return -1;
    const int64_t G = K / Q4O_GROUP;
    float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K + M * G + 1));
    float* xs = xf + M * K;
    for (int64_t i = 0; i < M * K; ++i) xf[i] = load_x(x, x_dtype, i);
    for (int64_t m = 0; m < M; ++m)
        for (int64_t g = 0; g < G; ++g) {
            float l[8] = {0};
            for (int j = 0; j < Q4O_GROUP; ++j) l[j & 7] = l[j & 7] + xf[m * K + g * Q4O_GROUP + j];
            xs[m * G + g] = lanes_sum8(l);
        }
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; ++n) {
        float q[Q4O_GROUP];
        float acc_y[64];
        for (int64_t m0 = 0; m0 < M; m0 += 64) {
            const int64_t mc = (M - m0) < 64 ? (M - m0) : 64;
            for (int64_t m = 0; m < mc; ++m) acc_y[m] = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                const uint32_t* wp = w->weight + n * (K / 8) + g * 8;
                for (int j = 0; j < Q4O_GROUP; ++j) q[j] = (float)((wp[j >> 3] >> (4 * (j & 7))) & 15u);
                const float s = q4o_bf16_to_f32(w->scales[n * G + g]);
                const float b = q4o_bf16_to_f32(w->biases[n * G + g]);
                for (int64_t m = 0; m < mc; ++m) {
                    const float* xp = xf + (m0 + m) * K + g * Q4O_GROUP;
                    float l[8] = {0};
                    for (int j = 0; j < Q4O_GROUP; j += 8)
                        for (int e = 0; e < 8; ++e) l[e] = l[e] + xp[j + e] * q[j + e];
                    const float acc = lanes_sum8(l);
                    const float t1 = s * acc;
                    const float t2 = b * xs[(m0 + m) * G + g];
                    acc_y[m] = acc_y[m] + (t1 + t2);
                }
            }
            for (int64_t m = 0; m < mc; ++m) y32[(m0 + m) * N + n] = acc_y[m];
        }
    }
    free(xf);
    return 0;
}

/* ---- RMSNorm (src/model/marlin.cpp:12-16) ------------------------------------------------------
 * bf16 x:  sq = bf16(x*x); var = bf16(sum(sq)) * 2^-log2(H) [bf16 mean]; the sum accumulates in
 *          binary32 (eight lanes) and rounds once to bf16.
 * f32 x:   sq = x*x; var = sum(sq) * (float)(1/H).
 * Then (both): r = 1 / sqrt(var + eps); y = (x * r) * (1 + w), binary32 — `variance + eps` with a
 * C++ float eps (src/core/config.h:20) and `1.0f + weight` promote to float32 in MLX's C++ API. */
void q4o_rms_norm(const void* x, int x_dtype, const uint16_t* w, int64_t M, int64_t H, float eps,
                  float* out) {
    for (int64_t m = 0; m < M; ++m) {
        float l[8] = {0};
        for (int64_t k = 0; k < H; ++k) {
            float v = load_x(x, x_dtype, m * H + k);
            float sq = v * v;
            if (x_dtype == Q4O_BF16) sq = bf16_round(sq);
            l[k & 7] = l[k & 7] + sq;
        }
        float sum = lanes_sum8(l);
        float var;
        if (x_dtype == Q4O_BF16) {
            var = bf16_round(bf16_round(sum) * bf16_round((float)(1.0 / (double)H)));
        } else {
            var = sum * (float)(1.0 / (double)H);
        }
        const float r = 1.0f / sqrtf(var + eps);
        for (int64_t k = 0; k < H; ++k) {
            float v = load_x(x, x_dtype, m * H + k);
            float a = v * r;
            float c = 1.0f + q4o_bf16_to_f32(w[k]);
            out[m * H + k] = a * c;
        }
    }
}

/* ---- SwiGLU (src/model/marlin.cpp:27-29): (sigmoid(g) * g) * u --------------------------------- */
static inline float sigmoidf_ref(float g) { return 1.0f / (1.0f + expf(-g)); }

void q4o_swiglu_f32(const float* g, const float* u, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float t = sigmoidf_ref(g[i]) * g[i];
        out[i] = t * u[i];
    }
}

void q4o_swiglu_bf16(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float gf = q4o_bf16_to_f32(g[i]);
        float sg = bf16_round(sigmoidf_ref(gf));
        float t = bf16_round(sg * gf);
        out[i] = q4o_f32_to_bf16(t * q4o_bf16_to_f32(u[i]));
    }
}

/* ---- MLP block (src/model/marlin.cpp:31-35) --------------------------------------------------- */
int q4o_mlp(const void* x, int x_dtype, int64_t M, const q4o_layer* L, void* y) {
    const int64_t I = L->gate.N, H = L->down.N;
    if (L->gate.K != L->up.K || L->up.N != I || L->down.K != I) return -1;
    float* g32 = (float*)malloc(sizeof(float) * (size_t)(3 * M * I + M * H + 1));
    float* u32 = g32 + M * I;
    float* a32 = u32 + M * I;
    float* o32 = a32 + M * I;
    if (q4o_qmatmul(x, x_dtype, M, &L->gate, g32) || q4o_qmatmul(x, x_dtype, M, &L->up, u32)) {
        free(g32);
        return -1;
    }
    int rc;
    if (x_dtype == Q4O_BF16) {
        uint16_t* gb = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)(3 * M * I + 1));
        uint16_t* ub = gb + M * I;
        uint16_t* ab = ub + M * I;
        for (int64_t i = 0; i < M * I; ++i) {
            gb[i] = q4o_f32_to_bf16(g32[i]);
            ub[i] = q4o_f32_to_bf16(u32[i]);
        }
        q4o_swiglu_bf16(gb, ub, ab, M * I);
        rc = q4o_qmatmul(ab, Q4O_BF16, M, &L->down, o32);
        for (int64_t i = 0; i < M * H; ++i) ((uint16_t*)y)[i] = q4o_f32_to_bf16(o32[i]);
        free(gb);
    } else {
        q4o_swiglu_f32(g32, u32, a32, M * I);
        rc = q4o_qmatmul(a32, Q4O_F32, M, &L->down, (float*)y);
    }
    free(g32);
    return rc;
}

/* ---- argmax (src/sampling/sampler.cpp:14-16) ------------------------------------------------- */
void q4o_argmax_f32(const float* logits, int64_t M, int64_t V, int32_t* ids, float* best) {
    for (int64_t m = 0; m < M; ++m) {
        int64_t bi = 0;
        float bv = logits[m * V];
        for (int64_t v = 1; v < V; ++v)
            if (logits[m * V + v] > bv) {
                bv = logits[m * V + v];
                bi = v;
            }
        ids[m] = (int32_t)bi;
        if (best) best[m] = bv;
    }
}

int q4o_lm_head_argmax(const void* h, int h_dtype, int64_t M, const q4o_tensor* lm, int32_t* ids,
                       float* best) {
    float* logits = (float*)malloc(sizeof(float) * (size_t)(M * lm->N + 1));
    int rc = q4o_qmatmul(h, h_dtype, M, lm, logits);
    if (!rc) {
        if (h_dtype == Q4O_BF16)
            for (int64_t i = 0; i < M * lm->N; ++i) logits[i] = bf16_round(logits[i]);
        q4o_argmax_f32(logits, M, lm->N, ids, best);
    }
    free(logits);
    return rc;
}

/* ---- decode step -------------------------------------------------------------------------------
 * src/model/marlin.cpp:103-146 restricted to the Q4 sublayers: per layer
 *   p = rms_norm(h, norm_l); h = h + mlp(p)          (:141-142)
 * then rms_norm(h, final_norm) (:145), lm_head (:161-169) and argmax (sampler.cpp:15).  h starts as
 * the bf16 embedding rows; rms_norm's output is float32 (see q4o_rms_norm), so the MLP, the
 * residual stream and the logits are float32 from the first layer on. */
int q4o_decode_step(const uint16_t* h0, int64_t M, int64_t H, int n_layers, const q4o_layer* layers,
                    const uint16_t* final_norm, const q4o_tensor* lm, float eps, float* h_out,
                    int32_t* ids, float* best) {
    float* p = (float*)malloc(sizeof(float) * (size_t)(2 * M * H + 1));
    float* y = p + M * H;
    for (int64_t i = 0; i < M * H; ++i) h_out[i] = q4o_bf16_to_f32(h0[i]);
    int rc = 0;
    for (int l = 0; l < n_layers && !rc; ++l) {
        if (l == 0)
            q4o_rms_norm(h0, Q4O_BF16, layers[l].norm, M, H, eps, p);
        else
            q4o_rms_norm(h_out, Q4O_F32, layers[l].norm, M, H, eps, p);
        rc = q4o_mlp(p, Q4O_F32, M, &layers[l], y);
        for (int64_t i = 0; i < M * H; ++i) h_out[i] = h_out[i] + y[i];
    }
    if (!rc) {
        q4o_rms_norm(h_out, Q4O_F32, final_norm, M, H, eps, p);
        rc = q4o_lm_head_argmax(p, Q4O_F32, M, lm, ids, best);
    }
    free(p);
    return rc;
}
