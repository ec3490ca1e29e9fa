"""GPU parity of the tensor-parallel decode step with in-kernel exchanges (marlin_q4_tp_decode_step,
marlin_q4.tp.FusedTPDecodeStep) on 2, 4 and 8 GPUs, one process per GPU, at the full config-5 shape
(24 layers, hidden 2048, intermediate 6144, vocabulary 248320): sharded weights (gate/up by rows,
down by K with zero padding to a multiple of 512 -- 768 -> 1024 columns at 8 ranks --, lm_head by
vocabulary rows), the per-layer all-reduce and the argmax merge done by the kernels over peer memory.
Rows 1, 8, 16 and 32 (16 and 32 run as 8-row chunks, each a full step with its own exchanges).
Checked: every rank ends with the same h and ids (sums in rank order), a second call reproduces the
first, and the result matches the unsharded single-GPU step (ids exact, h within 1e-5 of the row
maximum; the all-reduce changes the summation order of down_proj).
The same workers check the tensor-parallel prefill MLP (config 4, marlin_q4.tp.TPPrefillMLP: 2048
bf16 rows, tcgen05 GEMMs on the shards, NCCL all-reduce of the binary32 down_proj partials) against
the single-GPU mlp_forward: every rank holds the same bf16 output, within the path's tolerance of
the single-GPU one and equal to it in nearly every element (only the rounding of sums that the
all-reduce ordered differently may move by one bf16 step).  Each world size is skipped on boxes
with fewer GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

H, I, V, NL = 2048, 6144, 248320, 24
ROWS = (1, 8, 16, 32)
PREFILL_ROWS = 2048


def _ngpu() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _model(mq):
    layers = []
    for l in range(NL):
        g = mq.quantize_weight(mq.synth_bf16((I, H), 1000 + 4 * l, 0.0, 0.02))
        u = mq.quantize_weight(mq.synth_bf16((I, H), 1001 + 4 * l, 0.0, 0.02))
        d = mq.quantize_weight(mq.synth_bf16((H, I), 1002 + 4 * l, 0.0, 0.02))
        layers.append(mq.Layer(mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02), g, u, d))
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 2000, 0.0, 0.02))
    fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
    return layers, lm, fn


def _worker(rank, world, port, path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", rank))
    steps = []
    try:
        import marlin_q4 as mq
        from marlin_q4 import tp
        layers, lm, fn = _model(mq)
        shards = [tp.shard_layer(L, rank, world, k_multiple=512) for L in layers]
        lm_s, off = tp.shard_vocab(lm, rank, world)
        res = {}
        for m in ROWS:
            h0 = mq.synth_bf16((m, H), 4000 + m, 0.0, 1.0)
            step = tp.FusedTPDecodeStep(shards, fn, lm_s, off, m)
            steps.append(step)
            ids, _, h = (t.clone() for t in step(h0))
            torch.cuda.synchronize()
            ids2, _, h2 = step(h0)
            torch.cuda.synchronize()
            same = bool(torch.equal(ids, ids2) and torch.equal(h, h2))
            err = mq.device_error()
            step.close()
            got = [None] * world
            dist.all_gather_object(got, (ids.cpu().numpy(), h.cpu().numpy()))
            across = all(np.array_equal(got[0][0], x[0]) and np.array_equal(got[0][1], x[1]) for x in got)
            if rank == 0:
                rids, _, rh = mq.DecodeStep(layers, fn, lm, m)(h0)
                torch.cuda.synchronize()
                rel = float(((h.float() - rh.float()).abs().max() / rh.float().abs().max()).item())
                res[f"ids{m}"] = ids.cpu().numpy()
                res[f"rids{m}"] = rids.cpu().numpy()
                res[f"rel{m}"] = rel
                res[f"same{m}"] = same
                res[f"err{m}"] = err
                res[f"across{m}"] = across
        # prefill MLP of layer 0 over the ranks
        xp = mq.synth_bf16((PREFILL_ROWS, H), 4500, 0.0, 1.0)
        pshard = tp.shard_layer(layers[0], rank, world, k_multiple=512, pad_gate_up=True)
        y = tp.TPPrefillMLP(pshard, PREFILL_ROWS)(xp).clone()
        torch.cuda.synchronize()
        got = [None] * world
        dist.all_gather_object(got, y.view(torch.int16).cpu().numpy())
        if rank == 0:
            L0 = layers[0]
            ry = mq.mlp_forward(xp, L0.gate_proj, L0.up_proj, L0.down_proj)
            torch.cuda.synchronize()
            yf, ryf = y.float(), ry.float()
            res["p_rel"] = float(((yf - ryf).abs().amax(dim=1) / ryf.abs().amax(dim=1)).max().item())
            res["p_eq"] = float((y.view(torch.int16) == ry.view(torch.int16)).float().mean().item())
            res["p_across"] = all(np.array_equal(got[0], g) for g in got)
            res["p_err"] = mq.device_error()
            np.savez(path, **res)
    finally:
        for st in steps:
            st.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_fused_step_matches_single_gpu(tmp_path, world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    path = str(tmp_path / "tp.npz")
    mp.spawn(_worker, args=(world, _free_port(), path), nprocs=world, join=True)
    r = np.load(path)
    for m in ROWS:
        assert int(r[f"err{m}"]) == 0, m
        assert bool(r[f"same{m}"]) and bool(r[f"across{m}"]), m
        assert np.array_equal(r[f"ids{m}"], r[f"rids{m}"]), m
        assert float(r[f"rel{m}"]) < 1e-5, m
    assert int(r["p_err"]) == 0
    assert bool(r["p_across"])
    assert float(r["p_rel"]) < 1e-2
    assert float(r["p_eq"]) > 0.9


def _padded_worker(rank, world, port, path, inter, pad_to, m):
    """One rank: the tensor-parallel entry with down_proj's K zero-padded from `inter` to `pad_to`
    columns (the layout of the 8-way shards, 768 -> 1024 columns) against the plain single-GPU step
    on the unpadded weights (for inter = 768, k % 512 != 0, that step runs the bf16 mma.sync family)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120))
    step = None
    try:
        import marlin_q4 as mq
        from marlin_q4 import tp
        layers, padded = [], []
        for l in range(3):
            g = mq.quantize_weight(mq.synth_bf16((inter, H), 1000 + 4 * l, 0.0, 0.02))
            u = mq.quantize_weight(mq.synth_bf16((inter, H), 1001 + 4 * l, 0.0, 0.02))
            d = mq.quantize_weight(mq.synth_bf16((H, inter), 1002 + 4 * l, 0.0, 0.02))
            nw = mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02)
            layers.append(mq.Layer(nw, g, u, d))
            padded.append(mq.Layer(nw, g, u, tp.pad_k(d, pad_to)))
        lm = mq.quantize_weight(mq.synth_bf16((16384, H), 2000, 0.0, 0.02))
        fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
        h0 = mq.synth_bf16((m, H), 4100, 0.0, 1.0)
        step = tp.FusedTPDecodeStep(padded, fn, lm, 0, m)
        ids, _, h = (t.clone() for t in step(h0))
        torch.cuda.synchronize()
        err = mq.device_error()
        step.close()
        step = None
        rids, _, rh = mq.DecodeStep(layers, fn, lm, m)(h0)
        torch.cuda.synchronize()
        rel = float(((h.float() - rh.float()).abs().max() / rh.float().abs().max()).item())
        np.savez(path, ids=ids.cpu().numpy(), rids=rids.cpu().numpy(), rel=rel, err=err)
    finally:
        if step is not None:
            step.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("inter,pad_to,m", [(6144, 6656, 2), (768, 1024, 20)])
def test_tp_entry_one_rank_with_padded_down_k(tmp_path, inter, pad_to, m):
    """20 rows run as two 8-row chunks and a 4-row chunk."""
    path = str(tmp_path / "pad.npz")
    mp.spawn(_padded_worker, args=(1, _free_port(), path, inter, pad_to, m), nprocs=1, join=True)
    r = np.load(path)
    assert int(r["err"]) == 0
    assert np.array_equal(r["ids"], r["rids"])
    assert float(r["rel"]) < 1e-5
