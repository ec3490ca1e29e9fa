"""GPU parity of the tensor-parallel decode step with in-kernel exchanges (marlin_q4_tp_decode_step,
marlin_q4.tp.FusedTPDecodeStep) on 2 GPUs, one process per GPU: sharded weights (gate/up by rows,
down by K with zero padding to a multiple of 512, lm_head by vocabulary rows), the per-layer
all-reduce and the argmax merge done by the kernels over peer memory.  Checked: every rank ends
with the same h and ids (sums in rank order), a second call reproduces the first (the exchange
flags return to zero), and the result matches the unsharded single-GPU step (ids exact, h within
1e-5 of the row maximum; the all-reduce changes the summation order of down_proj).  Skipped on
boxes with fewer than 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
need2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")

H, I, V, NL = 2048, 6144, 16384, 3


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, path, m):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    step = None
    try:
        import marlin_q4 as mq
        from marlin_q4 import tp
        layers = []
        for l in range(NL):
            g = mq.quantize_weight(mq.synth_bf16((I, H), 1000 + 4 * l, 0.0, 0.02))
            u = mq.quantize_weight(mq.synth_bf16((I, H), 1001 + 4 * l, 0.0, 0.02))
            d = mq.quantize_weight(mq.synth_bf16((H, I), 1002 + 4 * l, 0.0, 0.02))
            layers.append(mq.Layer(mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02), g, u, d))
        lm = mq.quantize_weight(mq.synth_bf16((V, H), 2000, 0.0, 0.02))
        fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
        h0 = mq.synth_bf16((m, H), 4000 + m, 0.0, 1.0)
        shards = [tp.shard_layer(L, rank, world, k_multiple=512) for L in layers]
        lm_s, off = tp.shard_vocab(lm, rank, world)
        step = tp.FusedTPDecodeStep(shards, fn, lm_s, off, m)
        ids, _, h = (t.clone() for t in step(h0))
        torch.cuda.synchronize()
        ids2, _, h2 = step(h0)
        torch.cuda.synchronize()
        same = bool(torch.equal(ids, ids2) and torch.equal(h, h2))
        err = mq.device_error()
        step.close()
        step = None
        got = [None] * world
        dist.all_gather_object(got, (ids.cpu().numpy(), h.cpu().numpy()))
        across = all(np.array_equal(got[0][0], x[0]) and np.array_equal(got[0][1], x[1]) for x in got)
        if rank == 0:
            ref = mq.DecodeStep(layers, fn, lm, m)
            rids, _, rh = ref(h0)
            torch.cuda.synchronize()
            rel = float(((h.float() - rh.float()).abs().max() / rh.float().abs().max()).item())
            np.savez(path, ids=ids.cpu().numpy(), rids=rids.cpu().numpy(), rel=rel, same=same, err=err,
                     across=across)
    finally:
        if step is not None:
            step.close()
        dist.destroy_process_group()


@need2
@pytest.mark.parametrize("m", [1, 4])
def test_tp2_fused_step_matches_single_gpu(tmp_path, m):
    path = str(tmp_path / "tp.npz")
    mp.spawn(_worker, args=(2, _free_port(), path, m), nprocs=2, join=True)
    r = np.load(path)
    assert int(r["err"]) == 0
    assert bool(r["same"]) and bool(r["across"])
    assert np.array_equal(r["ids"], r["rids"])
    assert float(r["rel"]) < 1e-5


def _padded_worker(rank, world, port, path):
    """One rank: the tensor-parallel entry with down_proj's K zero-padded by 512 columns (the layout
    the 8-way shards of a 6144-wide intermediate use) against the plain single-GPU step."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120))
    step = None
    try:
        import marlin_q4 as mq
        from marlin_q4 import tp
        layers, padded = [], []
        for l in range(NL):
            g = mq.quantize_weight(mq.synth_bf16((I, H), 1000 + 4 * l, 0.0, 0.02))
            u = mq.quantize_weight(mq.synth_bf16((I, H), 1001 + 4 * l, 0.0, 0.02))
            d = mq.quantize_weight(mq.synth_bf16((H, I), 1002 + 4 * l, 0.0, 0.02))
            nw = mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02)
            layers.append(mq.Layer(nw, g, u, d))
            padded.append(mq.Layer(nw, g, u, tp.pad_k(d, I + 512)))
        lm = mq.quantize_weight(mq.synth_bf16((V, H), 2000, 0.0, 0.02))
        fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
        h0 = mq.synth_bf16((2, H), 4100, 0.0, 1.0)
        step = tp.FusedTPDecodeStep(padded, fn, lm, 0, 2)
        ids, _, h = (t.clone() for t in step(h0))
        torch.cuda.synchronize()
        err = mq.device_error()
        step.close()
        step = None
        rids, _, rh = mq.DecodeStep(layers, fn, lm, 2)(h0)
        torch.cuda.synchronize()
        rel = float(((h.float() - rh.float()).abs().max() / rh.float().abs().max()).item())
        np.savez(path, ids=ids.cpu().numpy(), rids=rids.cpu().numpy(), rel=rel, err=err)
    finally:
        if step is not None:
            step.close()
        dist.destroy_process_group()


def test_tp_entry_one_rank_with_padded_down_k(tmp_path):
    path = str(tmp_path / "pad.npz")
    mp.spawn(_padded_worker, args=(1, _free_port(), path), nprocs=1, join=True)
    r = np.load(path)
    assert int(r["err"]) == 0
    assert np.array_equal(r["ids"], r["rids"])
    assert float(r["rel"]) < 1e-6
