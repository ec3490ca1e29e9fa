/*
 * marlin_q4.h — C ABI of the B200 (sm_100a) Q4 path of marlin-mlx.
 *
 * The reference (marlin-mlx) quantizes the SwiGLU MLP projections and the tied lm_head to MLX's
 * group-affine 4-bit format at load time and runs them through mx::quantized_matmul; greedy decode
 * takes mx::argmax of the logits.  The entry points below are what the reference's C++ model code
 * binds to replace those MLX calls; each cites the reference call site it stands in for
 * (paths relative to the marlin-mlx source tree).
 *
 * Conventions
 *   - All tensors are caller-owned DEVICE buffers (plain pointers); the library allocates nothing.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are stream-ordered and
 *     asynchronous: no host synchronisation happens inside any entry point.
 *   - bf16 values travel as uint16_t bit patterns.  Activation dtypes: MARLIN_Q4_BF16 (bf16) or
 *     MARLIN_Q4_F32 (IEEE binary32).  Every operator returns its result in the activation dtype,
 *     as MLX's type promotion does for bf16 scales/biases (bf16 x -> bf16 y, f32 x -> f32 y).
 *   - Q4 format (MLX layout, transpose=true): weight uint32 [n, k/8], element j of each run of 8
 *     in bits [4j, 4j+4); scales, biases bf16 [n, k/64]; w ~= scale * q + bias per 64-group.
 *   - Return value: MARLIN_Q4_OK (0) or a negative MARLIN_Q4_ERR_* code.  No C++ exception crosses
 *     this boundary.  Argument errors are detected before any launch.
 */
#ifndef MARLIN_Q4_H
#define MARLIN_Q4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MARLIN_Q4_OK 0
#define MARLIN_Q4_ERR_ARG (-1)         /* null pointer, negative or zero size, bad dtype */
#define MARLIN_Q4_ERR_SHAPE (-2)       /* k % 64 != 0, group_size != 64, bits != 4, mismatched dims */
#define MARLIN_Q4_ERR_ALIGN (-3)       /* a pointer is not aligned as the call requires (16 B) */
#define MARLIN_Q4_ERR_UNSUPPORTED (-4) /* a size outside what the kernels implement */
#define MARLIN_Q4_ERR_CUDA (-5)        /* a kernel launch failed (see marlin_q4_last_cuda_error) */
#define MARLIN_Q4_ERR_WORKSPACE (-6)   /* workspace missing, too small or misaligned */

#define MARLIN_Q4_BF16 0
#define MARLIN_Q4_F32 1

/* Device view of the reference's QuantizedTensor (src/core/types.h:75-82): the three MLX arrays
 * plus group_size (must be 64) and bits (must be 4).  weight, scales, biases: 16-byte aligned. */
typedef struct marlin_q4_tensor {
    const uint32_t* weight; /* [n, k/8] */
    const uint16_t* scales; /* bf16 [n, k/64] */
    const uint16_t* biases; /* bf16 [n, k/64] */
    int64_t n;              /* output features (rows) */
    int64_t k;              /* input features */
    int32_t group_size;
    int32_t bits;
} marlin_q4_tensor;

/* One decoder layer's Q4 path: the post-attention RMSNorm weight and the MLP projections
 * (src/model/marlin.h MLPWeights / LayerNormWeights, used at src/model/marlin.cpp:141-142). */
typedef struct marlin_q4_layer {
    const uint16_t* post_attn_norm; /* bf16 [hidden], offset weight (multiplier is 1 + w) */
    marlin_q4_tensor gate_proj;     /* [intermediate, hidden] */
    marlin_q4_tensor up_proj;       /* [intermediate, hidden] */
    marlin_q4_tensor down_proj;     /* [hidden, intermediate] */
} marlin_q4_layer;

/* ---- library ------------------------------------------------------------------------------- */
const char* marlin_q4_version(void);
const char* marlin_q4_status_string(int status);
/* cudaError_t of the last failed launch in this thread (0 if none). */
int marlin_q4_last_cuda_error(void);
/* Device-side error word of the current device (0 = none; 1 = a bounded wait timed out, on this
 * GPU's own copies or on a peer's exchange words; 3 = an embedding id out of range).
 * Synchronous: copies the word to the host.  clear != 0 resets it to 0.  While the word is set,
 * the exchange waits of marlin_q4_tp_decode_step return at once (see there): clear it before the
 * next step once the ranks are known to be in step again. */
int marlin_q4_device_error(int clear);
/* Bound of each wait for a peer GPU's exchange word in marlin_q4_tp_decode_step, in SM clock
 * cycles (process-wide, read when a step is issued; a step captured in a CUDA graph keeps the
 * value it was captured with).  0 restores the default, 4e9 cycles (about 2 s at 2 GHz). */
void marlin_q4_set_wait_limit_cycles(uint64_t cycles);
/* Programmatic dependent launch (kernels prefetch weights while their predecessor finishes).
 * Enabled by default; enable = 0 launches every kernel with plain stream ordering. */
void marlin_q4_set_pdl(int enable);
/* Decode kernel family (process-wide; both compute the same function, within the float tolerance,
 * and each is tested against the CPU checker; value 1 is not used):
 *   MARLIN_Q4_PATH_I8MMA   (default) integer tensor-core MMAs on the raw codes and 4 s8 activation
 *                          planes, exact int32 accumulation (k % 512 == 0, m <= 16 per launch);
 *                          the decode step's layers run on kernels that split K over thread-block
 *                          clusters and hand the activations over as ready-made operand planes;
 *   MARLIN_Q4_PATH_BF16MMA bf16 mma.sync on registers (any k % 64 == 0).
 * Shapes the integer-MMA family does not cover fall back to MARLIN_Q4_PATH_BF16MMA.  Returns
 * MARLIN_Q4_ERR_ARG for an unknown path. */
#define MARLIN_Q4_PATH_I8MMA 0
#define MARLIN_Q4_PATH_BF16MMA 2
int marlin_q4_set_decode_path(int path);
/* Kernels of the decode step's MLP layers with the integer-MMA family (process-wide):
 *   MARLIN_Q4_STEP_FUSED  (default) all layers in one persistent kernel: each CTA owns 64
 *                         intermediate features (gate/up rows, SwiGLU, their down_proj columns), the
 *                         activations meet in thread-block clusters, the down_proj partial rows add up
 *                         in a 64-bit fixed-point accumulator (order-independent, so deterministic),
 *                         and one arrival counter per layer orders the layers; serves hidden in
 *                         {512, 1024, 2048}, intermediate a multiple of 512 up to 64 x the SM count,
 *                         at most 24 layers, rows in chunks of 8;
 *   MARLIN_Q4_STEP_LAYERS two kernels per layer (K split over clusters, operand planes handed over).
 * Shapes the fused kernel does not serve run on the per-layer kernels.  Returns MARLIN_Q4_ERR_ARG
 * for an unknown value. */
#define MARLIN_Q4_STEP_FUSED 0
#define MARLIN_Q4_STEP_LAYERS 1
int marlin_q4_set_step_kernels(int which);
/* The kernels marlin_q4_decode_step runs, with the current settings on the current device, for m
 * rows of a model with the given hidden and intermediate sizes and n_layers layers of one shape:
 * MARLIN_Q4_STEP_FUSED or MARLIN_Q4_STEP_LAYERS (the latter also when the integer-MMA family is
 * off); MARLIN_Q4_ERR_ARG for a size below 1.  Queries the device (occupancy of the layer-stack
 * clusters) the first time; no launch. */
int marlin_q4_decode_step_kernels(int64_t m, int64_t hidden, int64_t intermediate, int32_t n_layers);

/* ---- quantize --------------------------------------------------------------------------------
 * Replaces mx::quantize(w, group_size, bits) at src/model/weights.cpp:46 (quantize_weight,
 * :45-56) and :183 (lm_head).  w: bf16 [n, k] row-major, 16-byte aligned.  Outputs wq [n, k/8],
 * scales/biases [n, k/64].  group_size must be 64 and bits 4 (the reference's only setting,
 * src/model/weights.cpp:45, src/core/types.h:79-80). */
int marlin_q4_quantize(const uint16_t* w, int64_t n, int64_t k, int32_t group_size, int32_t bits,
                       uint32_t* wq, uint16_t* scales, uint16_t* biases, void* stream);

/* ---- quantized matmul --------------------------------------------------------------------------
 * Replaces mx::quantized_matmul(x, w.weight, w.scales, w.biases, transpose=true, 64, 4) in
 * qmatmul (src/model/marlin.cpp:18-25; declared src/core/types.h:84) and MarlinModel::lm_head
 * (src/model/marlin.cpp:161-169).  x: [m, k] of x_dtype; y: [m, n] of x_dtype.  Any m >= 1.
 * bf16 x with m > 16 rows and k % 512 == 0 (prefill) runs one tcgen05 GEMM that dequantizes each
 * weight once to bf16 (s*q + b, one rounding) in shared memory; decode-sized m keeps every product
 * exact up to binary32 accumulation.  gate_up_swiglu and matmul_residual dispatch the same way. */
int marlin_q4_matmul(const void* x, int32_t x_dtype, int64_t m, const marlin_q4_tensor* w, void* y,
                     void* stream);

/* The same product with a binary32 result whatever x's dtype: the partial of a projection whose
 * input features are split across GPUs (the tensor-parallel down_proj of mlp_forward,
 * src/model/marlin.cpp:34), which the ranks sum before it is rounded to the activation dtype.
 * Dispatches like marlin_q4_matmul (bf16 x above 16 rows: the tcgen05 GEMM). */
int marlin_q4_matmul_f32(const void* x, int32_t x_dtype, int64_t m, const marlin_q4_tensor* w, float* y,
                         void* stream);
/* out[i] = bf16(x[i]) (round to nearest even): the summed binary32 partials back in the activation
 * dtype mlp_forward returns for bf16 x (src/model/marlin.cpp:31-35). */
int marlin_q4_cast_bf16(const float* x, int64_t count, uint16_t* out, void* stream);

/* ---- RMSNorm -------------------------------------------------------------------------------------
 * Replaces rms_norm (src/model/marlin.cpp:12-16): x * rsqrt(mean(x^2) + eps) * (1 + w), evaluated
 * as MLX's C++ API does with a float eps (src/core/config.h:20): the output is binary32. */
int marlin_q4_rms_norm(const void* x, int32_t x_dtype, const uint16_t* weight, int64_t m, int64_t h,
                       float eps, float* out, void* stream);

/* ---- MLP pieces -----------------------------------------------------------------------------------
 * gate/up projections + SwiGLU of mlp_forward (src/model/marlin.cpp:32-33 with swiglu :27-29),
 * optionally preceded by rms_norm (:141) when norm_weight != NULL (then the activation dtype is
 * binary32, as the norm's output is).  act: [m, gate->n] of the activation dtype. */
int marlin_q4_gate_up_swiglu(const void* x, int32_t x_dtype, int64_t m, const uint16_t* norm_weight,
                             float eps, const marlin_q4_tensor* gate, const marlin_q4_tensor* up,
                             void* act, void* stream);
/* down projection + residual (src/model/marlin.cpp:34 and :142): y = resid + act . W^T, binary32.
 * resid: [m, w->n] of resid_dtype; y: binary32 [m, w->n] (may alias resid when resid is binary32). */
int marlin_q4_matmul_residual(const void* act, int32_t act_dtype, int64_t m, const marlin_q4_tensor* w,
                              const void* resid, int32_t resid_dtype, float* y, void* stream);
/* Whole mlp_forward (src/model/marlin.cpp:31-35): y = down(swiglu(gate x, up x)), y in x_dtype.
 * workspace: >= marlin_q4_mlp_workspace_size bytes, 16-byte aligned. */
int marlin_q4_mlp(const void* x, int32_t x_dtype, int64_t m, const marlin_q4_tensor* gate,
                  const marlin_q4_tensor* up, const marlin_q4_tensor* down, void* y, void* workspace,
                  size_t workspace_bytes, void* stream);
size_t marlin_q4_mlp_workspace_size(int64_t m, int64_t intermediate, int32_t x_dtype);
/* out = h + y elementwise in binary32 (the residual add of src/model/marlin.cpp:142 after a
 * tensor-parallel all-reduce).  out may alias h when h is binary32. */
int marlin_q4_residual_add(const void* h, int32_t h_dtype, const float* y, int64_t count, float* out,
                           void* stream);

/* ---- lm_head + greedy argmax --------------------------------------------------------------------
 * Replaces MarlinModel::lm_head (src/model/marlin.cpp:161-169) followed by the greedy branch of
 * sample_token (src/sampling/sampler.cpp:14-16, mx::argmax: first index of the maximum), fused: the
 * logits are never written.  Optional final rms_norm (src/model/marlin.cpp:145) when
 * norm_weight != NULL.  The lm tensor may be a vocabulary shard whose row 0 is global index
 * vocab_offset.  Outputs (each optional, at least one): ids [m] (global index), best [m] (winning
 * logit, binary32), keys_out [m] (packed keys: (order-preserving logit bits << 32) | (2^32-1 - id),
 * so the max over shards of the keys is the global argmax with the reference's tie rule).
 * For bf16 hidden without norm, logits compare as bf16 (the operator's output dtype).
 * workspace: >= marlin_q4_lm_head_workspace_size(m) bytes, 16-byte aligned, zero-filled before the
 * first call; every call leaves it zeroed again. */
int marlin_q4_lm_head_argmax(const void* hidden, int32_t dtype, int64_t m, const uint16_t* norm_weight,
                             float eps, const marlin_q4_tensor* lm, int64_t vocab_offset, int32_t* ids,
                             float* best, uint64_t* keys_out, void* workspace, size_t workspace_bytes,
                             void* stream);
size_t marlin_q4_lm_head_workspace_size(int64_t m);

/* marlin_q4_lm_head_argmax without a workspace argument.  No counterpart in the reference: it
 * exists for callers that cannot allocate or own device scratch for this call, such as a binding
 * that replaces the lm_head + greedy sampling pair, whose call shape carries no buffer, or a
 * runtime that must not call cudaMalloc (a device-wide synchronisation) inside its decode loop.
 * Same arguments and results as marlin_q4_lm_head_argmax otherwise.
 * The keys live in one library-owned device array per device; each call first clears the part it
 * uses (cudaMemsetAsync on the caller's stream), so a call never depends on what an earlier call,
 * even an aborted one, left there.  Nothing is allocated.  m > MARLIN_Q4_LM_HEAD_STATIC_MAX_ROWS
 * returns MARLIN_Q4_ERR_UNSUPPORTED.  All calls on one device share that array: calls that can
 * overlap in time (different streams, unordered host threads) race and return wrong ids, so keep
 * them on one stream.  The first call on each device (and the first after the device's context has
 * been reset) looks the array up (cudaGetSymbolAddress) and must be made outside stream capture. */
#define MARLIN_Q4_LM_HEAD_STATIC_MAX_ROWS 64
int marlin_q4_lm_head_argmax_static(const void* hidden, int32_t dtype, int64_t m, const uint16_t* norm_weight,
                                    float eps, const marlin_q4_tensor* lm, int64_t vocab_offset, int32_t* ids,
                                    float* best, uint64_t* keys_out, void* stream);
/* ids/best from packed keys (after a cross-shard max-merge of keys_out). */
int marlin_q4_decode_keys(const uint64_t* keys, int64_t m, int32_t* ids, float* best, void* stream);

/* ---- decode step -----------------------------------------------------------------------------------
 * One greedy decode step over the Q4 path: text_forward_embeddings' layer loop restricted to the
 * Q4 sublayers (src/model/marlin.cpp:103-146: per layer h += mlp(rms_norm(h)); the mixer sublayers
 * are not part of this path), the final norm (:145), lm_head (:161-169) and argmax
 * (src/sampling/sampler.cpp:15).  h0: bf16 [m, hidden] embedding rows.  ids [m]; best [m]
 * (optional); h_out: binary32 [m, hidden] hidden state before the final norm (optional).
 * n_layers >= 1.
 * Runs as two kernels per layer plus the lm_head (more than 8 rows: in consecutive 8-row chunks,
 * each a full step; rows are independent).
 * workspace: >= marlin_q4_decode_step_workspace_size bytes, 256-byte aligned, zero-filled before
 * the first call (its head is left zeroed by every call); one workspace serves one (m, hidden,
 * intermediate) shape; zero it again before using it for another. */
int marlin_q4_decode_step(const uint16_t* h0, int64_t m, int64_t hidden, int32_t n_layers,
                          const marlin_q4_layer* layers, const uint16_t* final_norm, float eps,
                          const marlin_q4_tensor* lm, int32_t* ids, float* best, float* h_out,
                          void* workspace, size_t workspace_bytes, void* stream);
size_t marlin_q4_decode_step_workspace_size(int64_t m, int64_t hidden, int64_t intermediate);

/* ---- tensor-parallel decode step (no counterpart in the reference, which runs on one device) -----
 * The decode step of marlin_q4_decode_step over weights sharded across tp_size GPUs of one box, one
 * process per GPU: gate_proj/up_proj split by output rows, down_proj by input columns (its K may
 * carry zero padding up to a multiple of 512 beyond the rank's gate/up rows: zero codes, scales and
 * biases), the lm_head by vocabulary rows starting at vocab_offset.  The per-layer all-reduce of
 * the down_proj partial rows and the argmax merge happen inside the kernels over NVLink: every rank
 * stores its partial rows and keys, each value tagged with the step and layer in one 8-byte word,
 * into every rank's exchange buffer and waits (bounded, about 2 s, then records a device error) for
 * the others' words to carry the expected tag; sums run in rank order, so every rank holds the same
 * h and ids.  exchange[r]: rank r's exchange buffer as mapped in this process (the own one
 * from marlin_q4_device_alloc, the others from marlin_q4_ipc_open_handle), each
 * marlin_q4_tp_exchange_size bytes, zero before the first call (it then holds the rank's step
 * counter and the last values exchanged).  All ranks must call the step the same number of times,
 * at most 120 layers.  hidden a multiple of 512, down_proj K a multiple of 512; more than 8 rows
 * run as consecutive 8-row chunks, each a full step with its own exchanges.  workspace as for
 * marlin_q4_decode_step with intermediate = down_proj K.
 * A peer that stops writing (a dead rank): the first wait that runs out (marlin_q4_set_wait_limit_cycles)
 * sets device error 1 and every later exchange wait returns at once, so the step still completes,
 * its ids and h void; the host reads marlin_q4_device_error after the step.  The workspace keeps its
 * zero invariant through such a step. */
int marlin_q4_tp_decode_step(const uint16_t* h0, int64_t m, int64_t hidden, int32_t n_layers,
                             const marlin_q4_layer* layers, const uint16_t* final_norm, float eps,
                             const marlin_q4_tensor* lm_shard, int64_t vocab_offset, int32_t* ids, float* best,
                             float* h_out, int32_t tp_rank, int32_t tp_size, void* const* exchange, void* workspace,
                             size_t workspace_bytes, void* stream);
/* Bytes of one rank's exchange buffer (rows beyond 8 reuse the 8-row layout chunk by chunk). */
size_t marlin_q4_tp_exchange_size(int64_t m, int64_t hidden, int32_t tp);
/* Zero-filled device memory for an exchange buffer (cudaMalloc: its IPC handle covers exactly it). */
int marlin_q4_device_alloc(size_t bytes, void** ptr);
int marlin_q4_device_free(void* ptr);
/* CUDA IPC of an exchange buffer between the ranks' processes: handle = 64 bytes. */
int marlin_q4_ipc_get_handle(const void* ptr, void* handle);
int marlin_q4_ipc_open_handle(const void* handle, void** ptr);
int marlin_q4_ipc_close_handle(void* ptr);

/* ---- embedding rows from the tied Q4 table -------------------------------------------------------
 * MarlinModel::embed_tokens (src/model/marlin.cpp:63-65: mx::take(embed_tokens, ids, 0)) served from
 * the quantized lm_head it is tied to (src/model/weights.cpp:180-194, :207) instead of a separate
 * bf16 table: out[i, :] = bf16(scale * q + bias) of row ids[i], each element the exact value
 * rounded once (round to nearest even).  ids: int32 [m] on the device; out: bf16 [m, table->k],
 * 16-byte aligned.  An id outside [0, table->n) yields a zero row and device error 3. */
int marlin_q4_embed(const int32_t* ids, int64_t m, const marlin_q4_tensor* table, uint16_t* out, void* stream);

/* ---- synthetic inputs (benchmark / test support; no counterpart in the reference) ----------------
 * out[i] = bf16(mean + sigma * z_i), z_i a seeded Irwin-Hall(12) variate (mean 0, sd 1), the same
 * bit pattern the CPU checker produces for (seed, i). */
int marlin_q4_synth_bf16(uint16_t* out, int64_t n, uint64_t seed, float mean, float sigma, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MARLIN_Q4_H */
