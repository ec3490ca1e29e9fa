"""marlin_q4 — B200 (sm_100a) Q4 path of marlin-mlx: Python front end over libmarlin_q4.so.

The product is the CUDA library (marlin-mlx_b200/csrc, C ABI in include/marlin_q4.h); this
package binds it for torch tensors (tests, benchmarks, the tensor-parallel driver).
"""
from ._lib import LIB_PATH, MarlinQ4Error, load  # noqa: F401
from .ops import (DecodeStep, GreedyLoop, HostDecodeStep, Layer, LmHeadWorkspace, QuantizedTensor, cast_bf16, decode_keys,  # noqa: F401
                  device_error, embed_q4, gate_up_swiglu, lm_head_argmax, matmul_residual, mlp_forward,
                  matmul_f32, next_token_after_prefill, qmatmul, quantize_weight, residual_add, rms_norm, set_decode_path,
                  set_pdl, set_step_kernels, decode_step_kernels, synth_bf16)

__all__ = ["QuantizedTensor", "quantize_weight", "qmatmul", "matmul_f32", "cast_bf16", "rms_norm", "gate_up_swiglu", "matmul_residual",
           "mlp_forward", "residual_add", "lm_head_argmax", "LmHeadWorkspace", "decode_keys", "Layer",
           "DecodeStep", "GreedyLoop", "HostDecodeStep", "embed_q4", "next_token_after_prefill", "synth_bf16", "device_error", "set_pdl", "set_decode_path", "set_step_kernels", "decode_step_kernels", "load", "LIB_PATH", "MarlinQ4Error"]
