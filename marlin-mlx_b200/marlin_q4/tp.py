"""Tensor-parallel Q4 decode step: one process per GPU, torch.distributed (NCCL) for the exchange.

Sharding (the reference is single-device; this is the B200 multi-GPU layout of the same math):
  * gate_proj / up_proj column-parallel: rank r holds output rows [r*I/tp, (r+1)*I/tp) and computes
    its slice of SwiGLU locally (no communication);
  * down_proj row-parallel: rank r holds input columns [r*I/tp, ...) (64-aligned) and produces a
    binary32 partial [m, H] that one all-reduce(sum) per layer completes;
  * lm_head vocabulary-parallel: rank r holds rows [r*V/tp, ...); each rank reduces its shard to
    packed (logit, index) keys and one all-reduce(max) merges them, which equals the single-GPU
    argmax bit for bit (every logit is computed whole on one rank; ties keep the lowest index).

Keys are unsigned 64-bit; NCCL's max on int64 is signed, so keys travel XOR 2^63 (order-preserving
map from unsigned to signed).

The decode step, FusedTPDecodeStep, is marlin_q4_tp_decode_step: the down_proj kernel's epilogue
writes its partial rows into every rank's exchange buffer over NVLink and sums all ranks' rows
itself, and the lm_head kernel merges the keys the same way; the exchange buffers are mapped
between the processes with CUDA IPC (plain peer memory, no multicast).  No collective library call
per step.  (keys_to_signed serves a merge of packed keys through a signed all-reduce(max).)
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops
from ._lib import check
from ._lib import Q4Layer
from .ops import Layer, QuantizedTensor

SIGN = -(1 << 63)  # 0x8000000000000000 as int64


def pad_k(q: QuantizedTensor, k: int) -> QuantizedTensor:
    """The operand with its input features zero-padded to k (zero codes, scales and biases: the padded
    columns add exactly 0 whatever the activations there)."""
    if q.k == k:
        return q
    assert k > q.k and k % 64 == 0
    w = torch.zeros((q.n, k // 8), dtype=q.weight.dtype, device=q.weight.device)
    sc = torch.zeros((q.n, k // 64), dtype=q.scales.dtype, device=q.scales.device)
    bi = torch.zeros((q.n, k // 64), dtype=q.biases.dtype, device=q.biases.device)
    w[:, :q.k // 8] = q.weight
    sc[:, :q.k // 64] = q.scales
    bi[:, :q.k // 64] = q.biases
    return QuantizedTensor(w, sc, bi)


def pad_rows(q: QuantizedTensor, n: int) -> QuantizedTensor:
    """The operand with zero output rows appended up to n (zero codes, scales and biases: those
    outputs are exactly 0, and SwiGLU of a zero gate and up is exactly 0 too)."""
    if q.n == n:
        return q
    assert n > q.n
    w = torch.zeros((n, q.weight.shape[1]), dtype=q.weight.dtype, device=q.weight.device)
    sc = torch.zeros((n, q.scales.shape[1]), dtype=q.scales.dtype, device=q.scales.device)
    bi = torch.zeros((n, q.biases.shape[1]), dtype=q.biases.dtype, device=q.biases.device)
    w[:q.n] = q.weight
    sc[:q.n] = q.scales
    bi[:q.n] = q.biases
    return QuantizedTensor(w, sc, bi)


def shard_layer(layer: Layer, rank: int, world: int, k_multiple: int = 64, pad_gate_up: bool = False) -> Layer:
    """Rank `rank`'s shard of a layer; the down_proj shard's K is zero-padded to a multiple of
    `k_multiple` (512 for the kernels' tensor maps).  pad_gate_up: the gate/up shards get the same
    number of zero rows, so that their SwiGLU output already has the padded width (the prefill
    GEMM takes its input as it is; the decode step's planes leave the padding at zero itself)."""
    inter = layer.gate_proj.n
    assert inter % world == 0 and (inter // world) % 64 == 0, "intermediate must split into 64-aligned shards"
    r0, r1 = rank * inter // world, (rank + 1) * inter // world
    down = layer.down_proj.shard_k(r0, r1)
    down = pad_k(down, -(-down.k // k_multiple) * k_multiple)
    gate, up = layer.gate_proj.shard_rows(r0, r1), layer.up_proj.shard_rows(r0, r1)
    if pad_gate_up:
        gate, up = pad_rows(gate, down.k), pad_rows(up, down.k)
    return Layer(layer.post_attn_norm, gate, up, down)


def shard_vocab(lm: QuantizedTensor, rank: int, world: int) -> tuple[QuantizedTensor, int]:
    v = lm.n
    r0, r1 = rank * v // world, (rank + 1) * v // world
    return lm.shard_rows(r0, r1), r0


def keys_to_signed(keys: torch.Tensor) -> torch.Tensor:
    return torch.bitwise_xor(keys, SIGN)


class TPPrefillMLP:
    """mlp_forward (src/model/marlin.cpp:31-35) of a prefill block of rows over the ranks of `group`:
    rank r holds gate/up rows and down_proj input columns [r*I/tp, (r+1)*I/tp) (padded with zeros to
    a multiple of 512, shard_layer(..., k_multiple=512, pad_gate_up=True)).  Per call: gate/up +
    SwiGLU as one tcgen05 GEMM over the rank's rows (bf16 act, as the reference rounds it), down_proj
    as a tcgen05 GEMM with a binary32 partial, one all-reduce(sum) of the partials over NCCL, then
    the sum rounded to bf16 (the dtype mlp_forward returns).  Call under torch.cuda.graph() to
    capture the kernels and the collective together."""

    def __init__(self, layer_shard: Layer, m: int, group=None):
        self.layer, self.m, self.group = layer_shard, m, group
        dev = layer_shard.post_attn_norm.device
        self.act = torch.empty((m, layer_shard.gate_proj.n), dtype=torch.bfloat16, device=dev)
        self.part = torch.empty((m, layer_shard.down_proj.n), dtype=torch.float32, device=dev)
        self.y = torch.empty((m, layer_shard.down_proj.n), dtype=torch.bfloat16, device=dev)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        L = self.layer
        assert x.dtype == torch.bfloat16 and x.shape == (self.m, L.gate_proj.k)
        ops.gate_up_swiglu(x, L.gate_proj, L.up_proj, out=self.act)
        ops.matmul_f32(self.act, L.down_proj, out=self.part)
        dist.all_reduce(self.part, op=dist.ReduceOp.SUM, group=self.group)
        return ops.cast_bf16(self.part, out=self.y)


class FusedTPDecodeStep:
    """Tensor-parallel decode step with the exchanges inside the kernels (marlin_q4_tp_decode_step).

    Collective at construction: every rank allocates its exchange buffer, the IPC handles are
    all-gathered over `group` (any backend), each rank maps the others' buffers.  Every rank must
    then call the step the same number of times, and call close() (also collective) before the
    process group goes away.  Call under torch.cuda.graph() to capture the whole step."""

    def __init__(self, layers: list[Layer], final_norm: torch.Tensor, lm_shard: QuantizedTensor, vocab_offset: int,
                 m: int, group=None, eps: float = 1e-6):
        lib = _lib.load()
        self.layers, self.final_norm, self.lm, self.off, self.m, self.eps = layers, final_norm, lm_shard, vocab_offset, m, eps
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        dev = final_norm.device
        self.hidden = lm_shard.k
        inter = layers[0].down_proj.k
        self.xbytes = lib.marlin_q4_tp_exchange_size(m, self.hidden, self.world)
        own = ctypes.c_void_p()
        check(lib.marlin_q4_device_alloc(self.xbytes, ctypes.byref(own)), "marlin_q4_device_alloc")
        self.own = own.value
        handle = ctypes.create_string_buffer(64)
        check(lib.marlin_q4_ipc_get_handle(own, handle), "marlin_q4_ipc_get_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        ptrs, self.opened = [], []
        for r, hb in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            check(lib.marlin_q4_ipc_open_handle(ctypes.create_string_buffer(hb, 64), ctypes.byref(p)),
                  "marlin_q4_ipc_open_handle")
            ptrs.append(p.value)
            self.opened.append(p.value)
        self.exchange = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)
        self.ws_bytes = lib.marlin_q4_decode_step_workspace_size(m, self.hidden, inter)
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.c_layers = (Q4Layer * len(layers))(*[L.c() for L in layers])
        self.c_lm = lm_shard.c()
        self.ids = torch.empty(m, dtype=torch.int32, device=dev)
        self.best = torch.empty(m, dtype=torch.float32, device=dev)
        self.h = torch.empty((m, self.hidden), dtype=torch.float32, device=dev)

    def __call__(self, h0: torch.Tensor):
        assert h0.dtype == torch.bfloat16 and h0.shape == (self.m, self.hidden)
        check(_lib.load().marlin_q4_tp_decode_step(
            h0.data_ptr(), self.m, self.hidden, len(self.layers), self.c_layers, self.final_norm.data_ptr(), self.eps,
            ctypes.byref(self.c_lm), self.off, self.ids.data_ptr(), self.best.data_ptr(), self.h.data_ptr(), self.rank,
            self.world, self.exchange, self.ws.data_ptr(), self.ws_bytes, ops._stream()), "marlin_q4_tp_decode_step")
        return self.ids, self.best, self.h

    def close(self):
        """Collective: unmap the peers' buffers and free the own one once no rank uses them."""
        if self.own is None:
            return
        lib = _lib.load()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            check(lib.marlin_q4_ipc_close_handle(ctypes.c_void_p(p)), "marlin_q4_ipc_close_handle")
        dist.barrier(group=self.group)
        check(lib.marlin_q4_device_free(ctypes.c_void_p(self.own)), "marlin_q4_device_free")
        self.own, self.opened = None, []
