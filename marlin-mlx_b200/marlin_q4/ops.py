"""Torch-tensor front end over the C ABI, mirroring the reference's operator surface.

Names follow marlin-mlx: ``QuantizedTensor`` (src/core/types.h:75-82), ``quantize_weight``
(src/model/weights.cpp:45-56), ``qmatmul`` (src/model/marlin.cpp:18-25), ``rms_norm`` (:12-16),
``mlp_forward`` (:31-35), ``lm_head`` + greedy ``sample_token`` (:161-169, sampler.cpp:9-16).
Tensors are CUDA tensors; every op launches on torch's current stream and goes through
libmarlin_q4.so — there is no PyTorch or CPU fallback.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import BF16, F32, Q4Layer, Q4Tensor, check


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    raise TypeError(f"activation dtype must be bfloat16 or float32, got {t.dtype}")


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


@dataclass
class QuantizedTensor:
    """MLX Q4 operand: weight uint32 [n, k/8] (held as int32 bits), scales/biases bf16 [n, k/64]."""
    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group_size: int = 64
    bits: int = 4
    quantized: bool = True

    @property
    def n(self) -> int:
        return self.weight.shape[0]

    @property
    def k(self) -> int:
        return self.weight.shape[1] * 8

    def c(self) -> Q4Tensor:
        return Q4Tensor(self.weight.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(), self.n, self.k,
                        self.group_size, self.bits)

    def shard_rows(self, r0: int, r1: int) -> "QuantizedTensor":
        """Rows [r0, r1) (output features) — a column-parallel / vocabulary shard."""
        return QuantizedTensor(self.weight[r0:r1].contiguous(), self.scales[r0:r1].contiguous(),
                               self.biases[r0:r1].contiguous())

    def shard_k(self, k0: int, k1: int) -> "QuantizedTensor":
        """Input features [k0, k1) (must be 64-aligned) — a row-parallel shard."""
        assert k0 % 64 == 0 and k1 % 64 == 0
        return QuantizedTensor(self.weight[:, k0 // 8:k1 // 8].contiguous(),
                               self.scales[:, k0 // 64:k1 // 64].contiguous(),
                               self.biases[:, k0 // 64:k1 // 64].contiguous())


def quantize_weight(w: torch.Tensor, bits: int = 4, group_size: int = 64) -> QuantizedTensor:
    """mx::quantize(w, group_size, bits) (src/model/weights.cpp:45-56)."""
    _cuda(w, "w")
    if w.dtype != torch.bfloat16 or w.dim() != 2:
        raise TypeError("w must be a 2-D bfloat16 tensor")
    n, k = w.shape
    wq = torch.empty((n, max(k // 8, 1)), dtype=torch.int32, device=w.device)
    s = torch.empty((n, max(k // 64, 1)), dtype=torch.bfloat16, device=w.device)
    b = torch.empty_like(s)
    check(_lib.load().marlin_q4_quantize(w.data_ptr(), n, k, group_size, bits, wq.data_ptr(), s.data_ptr(),
                                         b.data_ptr(), _stream()), "marlin_q4_quantize")
    return QuantizedTensor(wq, s, b, group_size, bits)


def qmatmul(x: torch.Tensor, w: QuantizedTensor) -> torch.Tensor:
    """mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4): [.., k] -> [.., n]."""
    _cuda(x, "x")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    y = torch.empty((x2.shape[0], w.n), dtype=x.dtype, device=x.device)
    tw = w.c()
    check(_lib.load().marlin_q4_matmul(x2.data_ptr(), _dtype_code(x), x2.shape[0], ctypes.byref(tw), y.data_ptr(),
                                       _stream()), "marlin_q4_matmul")
    return y.reshape(*lead, w.n)


def matmul_f32(x: torch.Tensor, w: QuantizedTensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x . dequant(W)^T with a binary32 result (the partial of a K-split projection): [m, k] -> [m, n]."""
    _cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    if out is None:
        out = torch.empty((x2.shape[0], w.n), dtype=torch.float32, device=x.device)
    tw = w.c()
    check(_lib.load().marlin_q4_matmul_f32(x2.data_ptr(), _dtype_code(x), x2.shape[0], ctypes.byref(tw),
                                           out.data_ptr(), _stream()), "marlin_q4_matmul_f32")
    return out


def cast_bf16(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16(x) of a binary32 tensor, round to nearest even (marlin_q4_cast_bf16)."""
    _cuda(x, "x")
    assert x.dtype == torch.float32
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    check(_lib.load().marlin_q4_cast_bf16(x.data_ptr(), x.numel(), out.data_ptr(), _stream()), "marlin_q4_cast_bf16")
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """rms_norm (src/model/marlin.cpp:12-16) with a float eps: binary32 output."""
    _cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    out = torch.empty(x2.shape, dtype=torch.float32, device=x.device)
    check(_lib.load().marlin_q4_rms_norm(x2.data_ptr(), _dtype_code(x), weight.data_ptr(), x2.shape[0],
                                         x2.shape[1], eps, out.data_ptr(), _stream()), "marlin_q4_rms_norm")
    return out.reshape(x.shape)


def gate_up_swiglu(x: torch.Tensor, gate: QuantizedTensor, up: QuantizedTensor,
                   norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    _cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    act_dtype = torch.float32 if norm_weight is not None else x.dtype
    if out is None:
        out = torch.empty((x2.shape[0], gate.n), dtype=act_dtype, device=x.device)
    tg, tu = gate.c(), up.c()
    check(_lib.load().marlin_q4_gate_up_swiglu(
        x2.data_ptr(), _dtype_code(x), x2.shape[0], norm_weight.data_ptr() if norm_weight is not None else None, eps,
        ctypes.byref(tg), ctypes.byref(tu), out.data_ptr(), _stream()), "marlin_q4_gate_up_swiglu")
    return out


def matmul_residual(act: torch.Tensor, w: QuantizedTensor, resid: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    m = act.reshape(-1, act.shape[-1]).shape[0]
    if out is None:
        out = torch.empty((m, w.n), dtype=torch.float32, device=act.device)
    tw = w.c()
    check(_lib.load().marlin_q4_matmul_residual(act.data_ptr(), _dtype_code(act), m, ctypes.byref(tw),
                                                resid.data_ptr(), _dtype_code(resid), out.data_ptr(), _stream()),
          "marlin_q4_matmul_residual")
    return out


def mlp_forward(x: torch.Tensor, gate: QuantizedTensor, up: QuantizedTensor, down: QuantizedTensor) -> torch.Tensor:
    """mlp_forward (src/model/marlin.cpp:31-35): down(swiglu(gate x, up x)), output in x's dtype."""
    _cuda(x, "x")
    x2 = x.reshape(-1, x.shape[-1])
    m, dt = x2.shape[0], _dtype_code(x)
    lib = _lib.load()
    ws_bytes = lib.marlin_q4_mlp_workspace_size(m, gate.n, dt)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    y = torch.empty((m, down.n), dtype=x.dtype, device=x.device)
    tg, tu, td = gate.c(), up.c(), down.c()
    check(lib.marlin_q4_mlp(x2.data_ptr(), dt, m, ctypes.byref(tg), ctypes.byref(tu), ctypes.byref(td),
                            y.data_ptr(), ws.data_ptr(), ws_bytes, _stream()), "marlin_q4_mlp")
    return y.reshape(*x.shape[:-1], down.n)


def residual_add(h: torch.Tensor, y: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(h.shape, dtype=torch.float32, device=h.device)
    check(_lib.load().marlin_q4_residual_add(h.data_ptr(), _dtype_code(h), y.data_ptr(), h.numel(), out.data_ptr(),
                                             _stream()), "marlin_q4_residual_add")
    return out


class LmHeadWorkspace:
    """Zero-initialised keys + counter the fused lm_head/argmax needs (left zeroed by every call)."""

    def __init__(self, m: int, device):
        nbytes = _lib.load().marlin_q4_lm_head_workspace_size(m)
        self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.m = m


def lm_head_argmax(hidden: torch.Tensor, lm: QuantizedTensor, norm_weight: torch.Tensor | None = None,
                   eps: float = 1e-6, vocab_offset: int = 0, workspace: LmHeadWorkspace | None = None,
                   want_keys: bool = False):
    """lm_head (src/model/marlin.cpp:161-169) + greedy argmax (sampler.cpp:14-16), fused.

    Returns (ids int32 [m], best float32 [m]) or, with want_keys, the packed int64 keys [m]."""
    _cuda(hidden, "hidden")
    h2 = hidden.reshape(-1, hidden.shape[-1])
    m = h2.shape[0]
    if workspace is None or workspace.m < m:
        workspace = LmHeadWorkspace(m, hidden.device)
    ids = torch.empty(m, dtype=torch.int32, device=hidden.device)
    best = torch.empty(m, dtype=torch.float32, device=hidden.device)
    keys = torch.empty(m, dtype=torch.int64, device=hidden.device) if want_keys else None
    tl = lm.c()
    check(_lib.load().marlin_q4_lm_head_argmax(
        h2.data_ptr(), _dtype_code(hidden), m, norm_weight.data_ptr() if norm_weight is not None else None, eps,
        ctypes.byref(tl), vocab_offset, ids.data_ptr(), best.data_ptr(), keys.data_ptr() if keys is not None else None,
        workspace.buf.data_ptr(), workspace.buf.numel(), _stream()), "marlin_q4_lm_head_argmax")
    if want_keys:
        return keys
    return ids, best


def next_token_after_prefill(hidden: torch.Tensor, lm: QuantizedTensor, norm_weight: torch.Tensor | None = None,
                             eps: float = 1e-6, workspace: LmHeadWorkspace | None = None):
    """Greedy token that starts the decode loop after a prefill of S rows.

    The reference runs lm_head over all S rows of the prefill hidden state (src/core/engine.cpp:64)
    and sample_token keeps only the last position (src/sampling/sampler.cpp:10-15); only that row's
    logits matter, so this runs the final norm + fused lm_head/argmax on the last row alone (one
    GEMV over the 248K-row head instead of an S-row GEMM).  hidden: [S, H] or [1, S, H].
    Returns (ids int32 [1], best float32 [1])."""
    h2 = hidden.reshape(-1, hidden.shape[-1])
    return lm_head_argmax(h2[-1:], lm, norm_weight, eps, workspace=workspace)


def embed_q4(ids: torch.Tensor, table: QuantizedTensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Embedding rows from the tied Q4 table (marlin_q4_embed): bf16(s*q + b) of rows `ids`."""
    _cuda(ids, "ids")
    assert ids.dtype == torch.int32
    m = ids.numel()
    if out is None:
        out = torch.empty((m, table.k), dtype=torch.bfloat16, device=ids.device)
    tc = table.c()
    check(_lib.load().marlin_q4_embed(ids.data_ptr(), m, ctypes.byref(tc), out.data_ptr(), _stream()),
          "marlin_q4_embed")
    return out


def decode_keys(keys: torch.Tensor):
    m = keys.numel()
    ids = torch.empty(m, dtype=torch.int32, device=keys.device)
    best = torch.empty(m, dtype=torch.float32, device=keys.device)
    check(_lib.load().marlin_q4_decode_keys(keys.data_ptr(), m, ids.data_ptr(), best.data_ptr(), _stream()),
          "marlin_q4_decode_keys")
    return ids, best


@dataclass
class Layer:
    post_attn_norm: torch.Tensor
    gate_proj: QuantizedTensor
    up_proj: QuantizedTensor
    down_proj: QuantizedTensor

    def c(self) -> Q4Layer:
        return Q4Layer(self.post_attn_norm.data_ptr(), self.gate_proj.c(), self.up_proj.c(), self.down_proj.c())


class DecodeStep:
    """One greedy decode step over the Q4 path (marlin_q4_decode_step), with persistent workspace."""

    def __init__(self, layers: list[Layer], final_norm: torch.Tensor, lm: QuantizedTensor, m: int,
                 eps: float = 1e-6):
        self.layers, self.final_norm, self.lm, self.m, self.eps = layers, final_norm, lm, m, eps
        dev = final_norm.device
        self.hidden = lm.k
        inter = max(L.gate_proj.n for L in layers)
        lib = _lib.load()
        self.ws_bytes = lib.marlin_q4_decode_step_workspace_size(m, self.hidden, inter)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.c_layers = (Q4Layer * len(layers))(*[L.c() for L in layers])
        self.c_lm = lm.c()
        self.ids = torch.empty(m, dtype=torch.int32, device=dev)
        self.best = torch.empty(m, dtype=torch.float32, device=dev)
        self.h = torch.empty((m, self.hidden), dtype=torch.float32, device=dev)

    def __call__(self, h0: torch.Tensor):
        assert h0.dtype == torch.bfloat16 and h0.shape == (self.m, self.hidden)
        check(_lib.load().marlin_q4_decode_step(
            h0.data_ptr(), self.m, self.hidden, len(self.layers), self.c_layers, self.final_norm.data_ptr(), self.eps,
            ctypes.byref(self.c_lm), self.ids.data_ptr(), self.best.data_ptr(), self.h.data_ptr(), self.ws.data_ptr(),
            self.ws_bytes, _stream()), "marlin_q4_decode_step")
        return self.ids, self.best, self.h


class HostDecodeStep:
    """A decode step fed from, and read back into, pinned host buffers, for a serving loop whose
    embeddings come from and whose tokens go to the host: the copy of the embedding rows to the
    device, the step (a DecodeStep, or a tensor-parallel step with the same call) and the copy of
    its ids back are captured once as one CUDA graph, so each token costs one graph launch and one
    synchronisation instead of three stream operations and a synchronisation.  The reference's decode
    loop reads every token on the host the same way (`token.item()`, src/core/engine.cpp:80).

    h_host: pinned bf16 [m, hidden], refilled by the caller before each call; ids_host: pinned int32
    [m], valid when the call returns.  Both stay bound to the graph until close().  The constructor
    runs the step once, eagerly, on what h_host holds at that time (before the capture)."""

    def __init__(self, step, h_host: torch.Tensor, ids_host: torch.Tensor):
        m, hidden = step.m, step.hidden
        if not (h_host.is_pinned() and ids_host.is_pinned()):
            raise ValueError("h_host and ids_host must be pinned host tensors")
        if h_host.dtype != torch.bfloat16 or tuple(h_host.shape) != (m, hidden):
            raise ValueError(f"h_host must be bf16 [{m}, {hidden}]")
        if ids_host.dtype != torch.int32 or ids_host.numel() != m:
            raise ValueError(f"ids_host must be int32 [{m}]")
        self.step, self.h_host, self.ids_host = step, h_host, ids_host
        self.h0 = torch.empty((m, hidden), dtype=torch.bfloat16, device=step.ids.device)
        side = torch.cuda.Stream(device=self.h0.device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # one eager run first (library set-up outside the capture)
            self._body()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body()
        torch.cuda.current_stream().synchronize()

    def _body(self):
        self.h0.copy_(self.h_host, non_blocking=True)
        self.step(self.h0)
        self.ids_host.copy_(self.step.ids, non_blocking=True)

    def __call__(self) -> torch.Tensor:
        self.graph.replay()
        torch.cuda.current_stream().synchronize()
        return self.ids_host

    def close(self):
        self.graph = None


class GreedyLoop:
    """run_decode_loop's greedy path (src/core/engine.cpp:79-94) on the device: per token, the
    embedding rows of the current ids from the tied Q4 table (embed_q4), one DecodeStep, and its ids
    fed back, with no host synchronisation between tokens (the reference syncs every step, :80).
    Every kernel of one token is stream-ordered, so a caller may capture tokens in a CUDA graph."""

    def __init__(self, layers: list[Layer], final_norm: torch.Tensor, lm: QuantizedTensor, m: int,
                 eps: float = 1e-6):
        self.step = DecodeStep(layers, final_norm, lm, m, eps)
        self.lm = lm
        self.h0 = torch.empty((m, lm.k), dtype=torch.bfloat16, device=final_norm.device)

    def __call__(self, ids0: torch.Tensor, n_tokens: int) -> torch.Tensor:
        """ids0: int32 [m] on the device.  Returns int32 [n_tokens, m]: the ids of each step."""
        out = torch.empty((n_tokens, ids0.numel()), dtype=torch.int32, device=ids0.device)
        cur = ids0
        for t in range(n_tokens):
            embed_q4(cur, self.lm, out=self.h0)
            ids, _, _ = self.step(self.h0)
            out[t].copy_(ids)
            cur = out[t]
        return out


def synth_bf16(shape, seed: int, mean: float = 0.0, sigma: float = 1.0, device="cuda") -> torch.Tensor:
    """Seeded synthetic bf16 tensor (bit-identical to the CPU generator for the same seed)."""
    out = torch.empty(shape, dtype=torch.bfloat16, device=device)
    check(_lib.load().marlin_q4_synth_bf16(out.data_ptr(), out.numel(), seed, mean, sigma, _stream()),
          "marlin_q4_synth_bf16")
    return out


def device_error(clear: bool = True) -> int:
    return _lib.load().marlin_q4_device_error(1 if clear else 0)


def set_pdl(enable: bool) -> None:
    _lib.load().marlin_q4_set_pdl(1 if enable else 0)


DECODE_PATHS = {"i8": _lib.PATH_I8MMA, "bf16": _lib.PATH_BF16MMA}


def set_decode_path(path: str) -> None:
    """Select the decode kernel family: "i8" (integer MMAs, default: the decode step on the cluster
    K-split kernels with operand planes handed between them) or "bf16" (mma.sync)."""
    check(_lib.load().marlin_q4_set_decode_path(DECODE_PATHS[path]), "marlin_q4_set_decode_path")


STEP_KERNELS = {"fused": _lib.STEP_FUSED, "layers": _lib.STEP_LAYERS}


def set_step_kernels(which: str) -> None:
    """Select the kernels of the decode step's MLP layers: "fused" (default: all layers in one
    persistent kernel) or "layers" (two cluster split-K kernels per layer)."""
    check(_lib.load().marlin_q4_set_step_kernels(STEP_KERNELS[which]), "marlin_q4_set_step_kernels")


def decode_step_kernels(m: int, hidden: int, intermediate: int, n_layers: int) -> str:
    """Which kernels marlin_q4_decode_step runs for this shape here: "fused" or "layers"."""
    r = _lib.load().marlin_q4_decode_step_kernels(m, hidden, intermediate, n_layers)
    check(min(r, 0), "marlin_q4_decode_step_kernels")
    return "fused" if r == _lib.STEP_FUSED else "layers"
