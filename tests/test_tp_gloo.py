"""Tensor-parallel decode step on CPU ranks (gloo, world size 2): the sharding (marlin_q4/tp.py
shard_layer / shard_vocab, MLX layout slices of the Q4 operands) and the exchange protocol (one
all-reduce(sum) of binary32 partials per layer, one all-reduce(max) of packed argmax keys through
the signed XOR 2^63 map) reproduce the unsharded computation.  The per-rank math is the CPU
checker's, so the test needs no GPU; the GPU kernels run the same protocol under torchrun."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import q4_oracle as qo

H, I, V, NL, M = 256, 512, 1000, 2, 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _model(oracle):
    layers = []
    for l in range(NL):
        g = oracle.quantize(oracle.synth_bf16((I, H), 100 + l, 0.0, 0.05))
        u = oracle.quantize(oracle.synth_bf16((I, H), 200 + l, 0.0, 0.05))
        d = oracle.quantize(oracle.synth_bf16((H, I), 300 + l, 0.0, 0.05))
        nw = oracle.synth_bf16((H,), 400 + l, 0.1, 0.02)
        layers.append((nw, g, u, d))
    fn = oracle.synth_bf16((H,), 500, 0.1, 0.02)
    lm = oracle.quantize(oracle.synth_bf16((V, H), 600, 0.0, 0.05))
    h0 = oracle.synth_bf16((M, H), 700, 0.0, 1.0)
    return layers, fn, lm, h0


def _to_qt(q):
    from marlin_q4.ops import QuantizedTensor
    return QuantizedTensor(torch.from_numpy(q.weight.view(np.int32).copy()),
                           torch.from_numpy(q.scales.view(np.int16).copy()),
                           torch.from_numpy(q.biases.view(np.int16).copy()))


def _from_qt(t):
    return qo.Q4(t.weight.numpy().view(np.uint32), t.scales.numpy().view(np.uint16), t.biases.numpy().view(np.uint16))


def pack_keys(best: np.ndarray, ids: np.ndarray) -> np.ndarray:
    """(order-preserving logit bits << 32) | (2^32 - 1 - id): the lm_head kernels' key format."""
    u = best.astype(np.float32).view(np.uint32).astype(np.uint64)
    o = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000).astype(np.uint64)
    return ((o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - ids.astype(np.uint64))).view(np.int64)


def unpack_ids(keys: np.ndarray) -> np.ndarray:
    k = keys.view(np.uint64)
    return (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)


def _worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from marlin_q4 import tp
        from marlin_q4.ops import Layer
        oracle = qo.COracle()
        layers, fn, lm, h0 = _model(oracle)
        # shard with the product's helpers (torch CPU tensors in the MLX layout)
        shards = []
        for nw, g, u, d in layers:
            L = tp.shard_layer(Layer(torch.from_numpy(nw.view(np.int16)), _to_qt(g), _to_qt(u), _to_qt(d)), rank, world)
            shards.append((nw, _from_qt(L.gate_proj), _from_qt(L.up_proj), _from_qt(L.down_proj)))
        lm_shard, off = tp.shard_vocab(_to_qt(lm), rank, world)
        # the TP step: per layer norm -> local gate/up + SwiGLU -> partial down -> all-reduce(sum) -> residual
        cur = h0
        for nw, g, u, d in shards:
            x = oracle.rms_norm(cur, nw)
            act = oracle.swiglu_f32(oracle.qmatmul(x, g), oracle.qmatmul(x, u))
            part = torch.from_numpy(oracle.qmatmul(act, d))
            dist.all_reduce(part, op=dist.ReduceOp.SUM)
            base = qo.bf16_to_f32(cur) if cur.dtype == np.uint16 else cur
            cur = (base + part.numpy()).astype(np.float32)
        ids_l, best_l = oracle.lm_head_argmax(oracle.rms_norm(cur, fn), _from_qt(lm_shard))
        keys = torch.from_numpy(pack_keys(best_l, ids_l.astype(np.int64) + off))
        sk = tp.keys_to_signed(keys)
        dist.all_reduce(sk, op=dist.ReduceOp.MAX)
        ids = unpack_ids(tp.keys_to_signed(sk).numpy())
        if rank == 0:
            rids, rbest, rh = oracle.decode_step(h0, layers, fn, lm)
            err = float(np.abs(cur - rh).max() / np.abs(rh).max())
            np.savez(result_path, ids=ids, rids=rids, err=err)
    finally:
        dist.destroy_process_group()


def test_tp2_decode_step_matches_unsharded(tmp_path):
    path = str(tmp_path / "tp.npz")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    r = np.load(path)
    assert np.array_equal(r["ids"], r["rids"].astype(np.int64))
    assert float(r["err"]) < 1e-5


def test_key_merge_tie_takes_lowest_global_index():
    """Equal maxima on two shards: the max of the signed keys decodes to the lower global index."""
    from marlin_q4 import tp
    best = np.array([1.5, 1.5], np.float32)
    k_rank0 = torch.from_numpy(pack_keys(best[:1], np.array([700])))
    k_rank1 = torch.from_numpy(pack_keys(best[1:], np.array([12])))
    merged = torch.maximum(tp.keys_to_signed(k_rank0), tp.keys_to_signed(k_rank1))
    assert unpack_ids(tp.keys_to_signed(merged).numpy())[0] == 12
    # negative logits order correctly too
    neg = torch.from_numpy(pack_keys(np.array([-3.0, -0.5], np.float32), np.array([1, 2])))
    s = tp.keys_to_signed(neg)
    assert int(torch.argmax(s)) == 1
