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
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops
from .ops import Layer, QuantizedTensor

SIGN = -(1 << 63)  # 0x8000000000000000 as int64


def shard_layer(layer: Layer, rank: int, world: int) -> Layer:
    inter = layer.gate_proj.n
    assert inter % world == 0 and (inter // world) % 64 == 0, "intermediate must split into 64-aligned shards"
    r0, r1 = rank * inter // world, (rank + 1) * inter // world
    return Layer(layer.post_attn_norm, layer.gate_proj.shard_rows(r0, r1), layer.up_proj.shard_rows(r0, r1),
                 layer.down_proj.shard_k(r0, r1))


def shard_vocab(lm: QuantizedTensor, rank: int, world: int) -> tuple[QuantizedTensor, int]:
    v = lm.n
    r0, r1 = rank * v // world, (rank + 1) * v // world
    return lm.shard_rows(r0, r1), r0


def keys_to_signed(keys: torch.Tensor) -> torch.Tensor:
    return torch.bitwise_xor(keys, SIGN)


class TPDecodeStep:
    """Decode step over sharded weights.  Call under torch.cuda.graph() to capture all kernels and
    the NCCL collectives in one graph."""

    def __init__(self, layers: list[Layer], final_norm: torch.Tensor, lm_shard: QuantizedTensor, vocab_offset: int,
                 m: int, group=None, eps: float = 1e-6):
        self.layers, self.final_norm, self.lm, self.off, self.m, self.eps = layers, final_norm, lm_shard, vocab_offset, m, eps
        self.group = group
        dev = final_norm.device
        H = lm_shard.k
        inter = layers[0].gate_proj.n
        self.h = torch.empty((m, H), dtype=torch.float32, device=dev)
        self.partial = torch.empty((m, H), dtype=torch.float32, device=dev)
        self.act = torch.empty((m, inter), dtype=torch.float32, device=dev)
        self.ws = ops.LmHeadWorkspace(m, dev)
        self.keys = torch.empty(m, dtype=torch.int64, device=dev)

    def __call__(self, h0: torch.Tensor):
        cur = h0
        for L in self.layers:
            ops.gate_up_swiglu(cur, L.gate_proj, L.up_proj, norm_weight=L.post_attn_norm, eps=self.eps, out=self.act)
            y = ops.qmatmul(self.act, L.down_proj)  # binary32 partial of the row-parallel down_proj
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
            ops.residual_add(cur, y, out=self.h)
            cur = self.h
        keys = ops.lm_head_argmax(cur, self.lm, norm_weight=self.final_norm, eps=self.eps, vocab_offset=self.off,
                                  workspace=self.ws, want_keys=True)
        sk = keys_to_signed(keys)
        dist.all_reduce(sk, op=dist.ReduceOp.MAX, group=self.group)
        self.keys.copy_(keys_to_signed(sk))
        ids, best = ops.decode_keys(self.keys)
        return ids, best, self.h
