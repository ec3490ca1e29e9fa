/*
 * q4_oracle.h — CPU restatement of marlin-mlx's Q4 path.  TEST INFRASTRUCTURE ONLY.
 *
 * This oracle is the checker for the CUDA product in marlin-mlx_b200/.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.  The product never
 * links or calls it.
 *
 * PARITY UNPINNED.  The reference (marlin-mlx) delegates all Q4 arithmetic to MLX v0.25.2
 * (CMakeLists.txt:15-19, ml-explore/mlx tag v0.25.2), which is fetched at configure time and is
 * absent here; the reference ships no tests, fixtures or golden vectors for this path.  The
 * functions below restate MLX's published affine-quantization algorithm and the reference's
 * call-site composition (file:line cited per function); the choices MLX's documentation leaves
 * open are explicit flags (Q4O_*), with the default being this restatement's reading of the
 * MLX v0.25.2 GPU kernel the reference actually runs (mx::quantize on the default device).
 *
 * Bit patterns: bf16 values are passed as uint16_t.  All float arithmetic is IEEE binary32 with
 * round-to-nearest-even and no contraction (the Makefile passes -ffp-contract=off).
 */
#ifndef MARLIN_Q4_ORACLE_H
#define MARLIN_Q4_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q4O_GROUP 64
#define Q4O_BITS 4

/* Quantize switches (0 = default restatement). */
#define Q4O_ROUND_HALF_EVEN 1u   /* codes/q0 use rint (ties to even) instead of round (ties away) */
#define Q4O_TRUE_MINMAX 2u       /* group max starts at -inf instead of 0 */
#define Q4O_NO_ZERO_SNAP 4u      /* documented formula only: s=(max-min)/15, b=min, no edge snap */
#define Q4O_BF16_PARAMS_FIRST 8u /* round s,b to bf16 before computing the codes */

enum { Q4O_BF16 = 0, Q4O_F32 = 1 };

typedef struct {
    const uint32_t* weight; /* [N, K/8]  nibble j of word w = element 8w+j, bits [4j,4j+4) */
    const uint16_t* scales; /* bf16 [N, K/64] */
    const uint16_t* biases; /* bf16 [N, K/64] */
    int64_t N, K;
} q4o_tensor;

typedef struct {
    const uint16_t* norm; /* bf16 [H]  RMSNorm offset weight (multiplier is 1+w) */
    q4o_tensor gate;      /* [I, H] */
    q4o_tensor up;        /* [I, H] */
    q4o_tensor down;      /* [H, I] */
} q4o_layer;

/* ---- scalar helpers ---------------------------------------------------------------------- */
float q4o_bf16_to_f32(uint16_t h);
uint16_t q4o_f32_to_bf16(float f); /* round to nearest even */

/* ---- seeded synthetic generator ------------------------------------------------------------
 * Element i of stream `seed` is mean + sigma * z, z = (S - 393210) / 65536 where S is the sum of
 * twelve 16-bit lanes of three splitmix64 outputs (Irwin-Hall(12): mean 0, sd 1, |z| <= 6).
 * Integer sums, one product and one sum in binary32, then bf16 round-to-nearest-even: the GPU
 * generator in the product library reproduces it bit for bit. */
uint16_t q4o_synth_bf16_at(uint64_t seed, uint64_t i, float mean, float sigma);
void q4o_synth_bf16(uint16_t* out, int64_t n, uint64_t seed, float mean, float sigma);

/* ---- quantize ----------------------------------------------------------------------------- */
/* mx::quantize(w, 64, 4) as called at src/model/weights.cpp:46 and :183.  Returns 0 or -1 on a
 * bad shape (K % 64 != 0, group_size != 64, bits != 4).
 *
 * The reference calls mx::quantize on MLX's default device, the Apple GPU (src/model/weights.cpp:
 * 46-47 evaluates it right away; src/model/marlin.cpp:309-313 loads on that device), so the defaults
 * restate what this restatement takes MLX v0.25.2's GPU affine-quantize kernel to do.  Each default
 * is UNPINNED (no MLX here, no upstream vectors); each has a flag and a known-answer vector in
 * tests/golden/ that tells the two readings apart:
 *   - group maximum starts at 0, minimum at +inf (Q4O_TRUE_MINMAX starts the maximum at -inf):
 *     an all-negative group then snaps its bias to the minimum and its scale to a positive step;
 *   - round = ties away from zero, as Metal's round() is (Q4O_ROUND_HALF_EVEN: rint);
 *   - zero-point snap: s = edge / round(edge / s), b = edge, so the extreme of larger magnitude is
 *     exact (Q4O_NO_ZERO_SNAP: the documented s = (max - min) / 15, b = min);
 *   - codes from the binary32 scale and bias, which are then rounded to bf16 only to be stored (the
 *     kernel computes in float and casts on the store; Q4O_BF16_PARAMS_FIRST rounds them first:
 *     kat_param_order shows the codes that differ). */
int q4o_quantize(const uint16_t* w, int64_t N, int64_t K, int group_size, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases, unsigned flags);
/* dequantized value of element (n,k) in binary32: s*q + b */
float q4o_dequant_at(const q4o_tensor* t, int64_t n, int64_t k);

/* ---- quantized matmul ------------------------------------------------------------------------
 * mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) (src/model/marlin.cpp:20-22,
 * :164-166): y[m,n] = sum_g ( s[n,g] * sum_{k in g} x[m,k] q[n,k] + b[n,g] * sum_{k in g} x[m,k] ),
 * binary32 accumulation.  y32 receives the binary32 result; for bf16 x the operator's output is
 * q4o_f32_to_bf16(y32). */
int q4o_qmatmul(const void* x, int x_dtype, int64_t M, const q4o_tensor* w, float* y32);

/* ---- RMSNorm (src/model/marlin.cpp:12-16, eps = 1e-6f from src/core/config.h:20) ------------
 * x * rsqrt(mean(x^2) + eps) * (1 + w) as MLX's C++ API evaluates it: x^2 and mean in x's dtype,
 * then `+ eps` (a C++ float) and `1.0f + weight` promote to binary32.  Output is binary32. */
void q4o_rms_norm(const void* x, int x_dtype, const uint16_t* w, int64_t M, int64_t H, float eps,
                  float* out);

/* ---- SwiGLU (src/model/marlin.cpp:27-29): (sigmoid(g) * g) * u ------------------------------- */
void q4o_swiglu_f32(const float* g, const float* u, float* out, int64_t n);
void q4o_swiglu_bf16(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n);

/* ---- MLP block (src/model/marlin.cpp:31-35) ----------------------------------------------------
 * x_dtype bf16: gate/up/act/out rounded to bf16 at every op boundary (out is bf16 bits in y).
 * x_dtype f32: all binary32 (out is float in y). */
int q4o_mlp(const void* x, int x_dtype, int64_t M, const q4o_layer* L, void* y);

/* ---- argmax (src/sampling/sampler.cpp:14-16): first index of the maximum ------------------- */
void q4o_argmax_f32(const float* logits, int64_t M, int64_t V, int32_t* ids, float* best);
/* lm_head (src/model/marlin.cpp:161-169) then greedy argmax.  For bf16 hidden the logits are
 * rounded to bf16 before the comparison (the operator's output dtype). best[m] = winning logit. */
int q4o_lm_head_argmax(const void* h, int h_dtype, int64_t M, const q4o_tensor* lm, int32_t* ids,
                       float* best);

/* ---- decode step (src/model/marlin.cpp:103-146 with the mixer sublayers as identity, then
 * :161-169 and src/sampling/sampler.cpp:14-16).  h0: bf16 [M,H] embeddings.  h_out: binary32
 * [M,H] hidden state after the last residual (before the final norm).  ids: [M]. ---------------- */
int q4o_decode_step(const uint16_t* h0, int64_t M, int64_t H, int n_layers, const q4o_layer* layers,
                    const uint16_t* final_norm, const q4o_tensor* lm, float eps, float* h_out,
                    int32_t* ids, float* best);

int q4o_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
