"""Failure detection of the tensor-parallel exchange on one GPU, without a GPU fault.

marlin_q4_tp_decode_step waits, bounded, for every peer rank's tagged words.  Here rank 0 of a
2-rank step gets, as rank 1's exchange buffer, a second zeroed buffer on its own GPU that no rank
ever writes: the stand-in for a peer that died between steps.  Every exchange wait of the step (24
row sums per layer and the argmax key merge) must then run out.  With the wait limit set to about
1 ms, the first wait that runs out records device error 1 and every later one returns at once, so
the whole step comes back in far less than a second; the same workspace then serves a healthy step
whose ids equal the single-GPU step's (its zero invariant survived the aborted step)."""
import ctypes
import time

import pytest
import torch

import marlin_q4 as mq
from marlin_q4 import _lib
from marlin_q4._lib import Q4Layer

pytestmark = pytest.mark.gpu

H, I, V, NL, M = 2048, 1024, 4096, 3, 2
LIMIT_CYCLES = 2_000_000  # about 1 ms at 2 GHz


def _model():
    layers = []
    for l in range(NL):
        g = mq.quantize_weight(mq.synth_bf16((I, H), 500 + 4 * l, 0.0, 0.02))
        u = mq.quantize_weight(mq.synth_bf16((I, H), 501 + 4 * l, 0.0, 0.02))
        d = mq.quantize_weight(mq.synth_bf16((H, I), 502 + 4 * l, 0.0, 0.02))
        layers.append(mq.Layer(mq.synth_bf16((H,), 503 + 4 * l, 0.1, 0.02), g, u, d))
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 520, 0.0, 0.02))
    fn = mq.synth_bf16((H,), 521, 0.1, 0.02)
    return layers, lm, fn


def _tp_step(lib, layers, lm, fn, h0, tp, exchange, ws, ids, best, h):
    c_layers = (Q4Layer * len(layers))(*[L.c() for L in layers])
    c_lm = lm.c()
    ex = (ctypes.c_void_p * tp)(*[b.data_ptr() for b in exchange])
    return lib.marlin_q4_tp_decode_step(h0.data_ptr(), M, H, len(layers), c_layers, fn.data_ptr(), 1e-6,
                                        ctypes.byref(c_lm), 0, ids.data_ptr(), best.data_ptr(), h.data_ptr(), 0, tp,
                                        ex, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)


def test_dead_peer_wait_runs_out_and_step_returns():
    lib = _lib.load()
    layers, lm, fn = _model()
    h0 = mq.synth_bf16((M, H), 530, 0.0, 1.0)
    xbytes = lib.marlin_q4_tp_exchange_size(M, H, 2)
    own = torch.zeros(xbytes, dtype=torch.uint8, device="cuda")
    silent_peer = torch.zeros(xbytes, dtype=torch.uint8, device="cuda")  # nobody writes rank 1's words
    ws_bytes = lib.marlin_q4_decode_step_workspace_size(M, H, I)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    ids = torch.empty(M, dtype=torch.int32, device="cuda")
    best = torch.empty(M, dtype=torch.float32, device="cuda")
    h = torch.empty((M, H), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    assert mq.device_error(clear=True) == 0
    lib.marlin_q4_set_wait_limit_cycles(LIMIT_CYCLES)
    try:
        t0 = time.perf_counter()
        rc = _tp_step(lib, layers, lm, fn, h0, 2, [own, silent_peer], ws, ids, best, h)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    finally:
        lib.marlin_q4_set_wait_limit_cycles(0)
    assert rc == 0, lib.marlin_q4_status_string(rc)
    assert mq.device_error(clear=True) == 1  # the wait ran out and said so
    assert dt < 1.0, f"the aborted step took {dt:.3f} s"

    # the same workspace, now as a 1-rank step: its head (argmax keys, CTA counter) is zero again
    rc = _tp_step(lib, layers, lm, fn, h0, 1, [own], ws, ids, best, h)
    assert rc == 0
    rids, _, rh = mq.DecodeStep(layers, fn, lm, M)(h0)
    torch.cuda.synchronize()
    assert mq.device_error() == 0
    assert torch.equal(ids, rids)
    rel = float(((h - rh).abs().max() / rh.abs().max()).item())
    assert rel < 1e-6

