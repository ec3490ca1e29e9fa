"""GPU parity: the full Q4 decode stack (config 5) — 24 x [RMSNorm(1+w) -> Q4 MLP -> residual] ->
final RMSNorm -> Q4 lm_head -> argmax — against the CPU oracle, fed the GPU-quantized weights.

The step runs its MLP layers as one persistent kernel (above 8 rows in 8-row chunks); the per-layer
integer-MMA kernels that split K over clusters and the bf16 mma.sync family's composition of
single-op kernels are checked against it."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
from gpu_util import f32, host_q4, make_q4, max_rel_row_err, u16

pytestmark = pytest.mark.gpu

H, I, V, L = 2048, 6144, 248320, 24


@pytest.fixture(scope="module")
def model():
    layers, host_layers = [], []
    for l in range(L):
        g, _ = make_q4(I, H, 1000 + 4 * l)
        u, _ = make_q4(I, H, 1001 + 4 * l)
        d, _ = make_q4(H, I, 1002 + 4 * l)
        nw = mq.synth_bf16((H,), 1003 + 4 * l, 0.1, 0.02)
        layers.append(mq.Layer(nw, g, u, d))
        host_layers.append((u16(nw), host_q4(g), host_q4(u), host_q4(d)))
    lm, _ = make_q4(V, H, 2000)
    fn = mq.synth_bf16((H,), 2001, 0.1, 0.02)
    return layers, host_layers, lm, host_q4(lm), fn, u16(fn)


@pytest.mark.parametrize("m", [1, 2, 3, 8, 12, 16, 20, 32])
def test_decode_step_matches_oracle(oracle, model, m):
    layers, hl, lm, hlm, fn, hfn = model
    step = mq.DecodeStep(layers, fn, lm, m)
    h0 = mq.synth_bf16((m, H), 3000 + m, 0.0, 1.0)
    ids, best, h = step(h0)
    torch.cuda.synchronize()
    rids, rbest, rh = oracle.decode_step(u16(h0), hl, hfn, hlm)
    assert max_rel_row_err(f32(h), rh) < 1e-3
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert mq.device_error() == 0
    # deterministic across calls
    ids2, _, h2 = step(h0)
    assert torch.equal(ids2, ids) and torch.equal(h2, h)


@pytest.mark.parametrize("m", [1, 5, 8, 20])
def test_layer_kernels_step_matches_oracle(oracle, model, m):
    """The per-layer kernels (two cluster split-K launches per layer) against the oracle and against
    the one-kernel layer stack (the default)."""
    layers, hl, lm, hlm, fn, hfn = model
    h0 = mq.synth_bf16((m, H), 3400 + m, 0.0, 1.0)
    ids_f, _, h_f = (t.clone() for t in mq.DecodeStep(layers, fn, lm, m)(h0))
    mq.set_step_kernels("layers")
    try:
        ids, _, h = mq.DecodeStep(layers, fn, lm, m)(h0)
        torch.cuda.synchronize()
    finally:
        mq.set_step_kernels("fused")
    rids, _, rh = oracle.decode_step(u16(h0), hl, hfn, hlm)
    assert max_rel_row_err(f32(h), rh) < 1e-3
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert max_rel_row_err(f32(h_f), f32(h).astype(np.float64)) < 1e-5
    assert torch.equal(ids_f, ids)
    assert mq.device_error() == 0


def test_decode_step_in_cuda_graph(model):
    layers, _, lm, _, fn, _ = model
    step = mq.DecodeStep(layers, fn, lm, 1)
    h0 = mq.synth_bf16((1, H), 3100, 0.0, 1.0)
    ids_eager = step(h0)[0].clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(h0)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(h0)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(step.ids, ids_eager)


@pytest.mark.parametrize("m", [1, 5])
def test_bf16_family_step_matches_i8(model, m):
    """The bf16 mma.sync family (single-op kernels composed) against the integer-MMA step."""
    layers, _, lm, _, fn, _ = model
    h0 = mq.synth_bf16((m, H), 3200 + m, 0.0, 1.0)
    ids, _, h = (t.clone() for t in mq.DecodeStep(layers, fn, lm, m)(h0))
    mq.set_decode_path("bf16")
    try:
        ids_c, _, h_c = mq.DecodeStep(layers, fn, lm, m)(h0)
        torch.cuda.synchronize()
    finally:
        mq.set_decode_path("i8")
    assert max_rel_row_err(f32(h), f32(h_c).astype(np.float64)) < 1e-4
    assert torch.equal(ids, ids_c)
    assert mq.device_error() == 0


@pytest.mark.parametrize("nl", [1, 2])
def test_short_stacks(oracle, model, nl):
    layers, hl, lm, hlm, fn, hfn = model
    step = mq.DecodeStep(layers[:nl], fn, lm, 2)
    h0 = mq.synth_bf16((2, H), 3300 + nl, 0.0, 1.0)
    ids, _, h = step(h0)
    torch.cuda.synchronize()
    rids, _, rh = oracle.decode_step(u16(h0), hl[:nl], hfn, hlm)
    assert max_rel_row_err(f32(h), rh) < 1e-4
    assert np.array_equal(ids.cpu().numpy(), rids)
