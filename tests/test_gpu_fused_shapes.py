"""GPU parity: the one-kernel MLP layer stack (marlin_q4_decode_step's default on one GPU) at the
hidden sizes it serves besides C5's 2048 (512 and 1024, intermediate 4 x hidden), against the CPU
oracle and against the per-layer kernels, and the shapes for which the step picks it."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
from gpu_util import f32, host_q4, make_q4, max_rel_row_err, u16

pytestmark = pytest.mark.gpu

V, NL = 4096, 3


def build(H, I, seed):
    layers, host = [], []
    for l in range(NL):
        g, _ = make_q4(I, H, seed + 4 * l)
        u, _ = make_q4(I, H, seed + 1 + 4 * l)
        d, _ = make_q4(H, I, seed + 2 + 4 * l)
        nw = mq.synth_bf16((H,), seed + 3 + 4 * l, 0.1, 0.02)
        layers.append(mq.Layer(nw, g, u, d))
        host.append((u16(nw), host_q4(g), host_q4(u), host_q4(d)))
    lm, _ = make_q4(V, H, seed + 100)
    fn = mq.synth_bf16((H,), seed + 101, 0.1, 0.02)
    return layers, host, lm, host_q4(lm), fn, u16(fn)


@pytest.mark.parametrize("H", [512, 1024])
@pytest.mark.parametrize("m", [1, 2, 5, 8])
def test_layer_stack_shapes_match_oracle(oracle, H, m):
    I = 4 * H
    layers, hl, lm, hlm, fn, hfn = build(H, I, 5000 + H + m)
    assert mq.decode_step_kernels(m, H, I, NL) == "fused"
    h0 = mq.synth_bf16((m, H), 5100 + m, 0.0, 1.0)
    ids, _, h = (t.clone() for t in mq.DecodeStep(layers, fn, lm, m)(h0))
    torch.cuda.synchronize()
    assert mq.device_error() == 0
    rids, _, rh = oracle.decode_step(u16(h0), hl, hfn, hlm)
    assert max_rel_row_err(f32(h), rh) < 1e-4
    assert np.array_equal(ids.cpu().numpy(), rids)
    mq.set_step_kernels("layers")
    try:
        assert mq.decode_step_kernels(m, H, I, NL) == "layers"
        ids_l, _, h_l = mq.DecodeStep(layers, fn, lm, m)(h0)
        torch.cuda.synchronize()
    finally:
        mq.set_step_kernels("fused")
    assert torch.equal(ids_l, ids)
    assert max_rel_row_err(f32(h), f32(h_l).astype(np.float64)) < 1e-5


def test_step_kernel_choice():
    """C5 (hidden 2048, intermediate 6144, 24 layers) runs the layer stack at every row count (more
    than 8 rows in 8-row chunks); shapes outside its envelope run the per-layer kernels."""
    for m in (1, 2, 8, 9, 32):
        assert mq.decode_step_kernels(m, 2048, 6144, 24) == "fused"
    assert mq.decode_step_kernels(1, 2048, 6144, 25) == "layers"   # more than 24 layers
    assert mq.decode_step_kernels(1, 1536, 6144, 24) == "layers"   # hidden not 512 / 1024 / 2048
    assert mq.decode_step_kernels(1, 2048, 6400, 24) == "layers"   # intermediate not a multiple of 512
    mq.set_decode_path("bf16")
    try:
        assert mq.decode_step_kernels(1, 2048, 6144, 24) == "layers"
    finally:
        mq.set_decode_path("i8")


@pytest.mark.parametrize("H,I", [(1024, 512), (1024, 1536), (2048, 1024)])
@pytest.mark.parametrize("m", [1, 8])
@pytest.mark.parametrize("nl", [1, 2])
def test_layer_stack_cluster_counts(oracle, H, I, m, nl):
    """One, two and three clusters (intermediate 512, 1024, 1536: one to three contributions per
    accumulator word) and stacks whose final h sits in the second and third accumulator."""
    layers, hl, lm, hlm, fn, hfn = build(H, I, 6000 + H + I + m)
    layers, hl = layers[:nl], hl[:nl]
    assert mq.decode_step_kernels(m, H, I, nl) == "fused"
    h0 = mq.synth_bf16((m, H), 6100 + m + nl, 0.0, 1.0)
    ids, _, h = (t.clone() for t in mq.DecodeStep(layers, fn, lm, m)(h0))
    torch.cuda.synchronize()
    assert mq.device_error() == 0
    rids, _, rh = oracle.decode_step(u16(h0), hl, hfn, hlm)
    assert max_rel_row_err(f32(h), rh) < 1e-4
    assert np.array_equal(ids.cpu().numpy(), rids)


def test_host_decode_step_matches_device_step():
    """HostDecodeStep (copy in, step, copy out as one graph) returns the ids of DecodeStep for each
    refill of its host buffer."""
    H, m = 1024, 2
    layers, hl, lm, hlm, fn, hfn = build(H, 4 * H, 7000)
    h_host = torch.empty((m, H), dtype=torch.bfloat16).pin_memory()
    ids_host = torch.empty(m, dtype=torch.int32).pin_memory()
    hs = mq.HostDecodeStep(mq.DecodeStep(layers, fn, lm, m), h_host, ids_host)
    ref = mq.DecodeStep(layers, fn, lm, m)
    try:
        for seed in (7100, 7101, 7102):
            h0 = mq.synth_bf16((m, H), seed, 0.0, 1.0)
            h_host.copy_(h0.cpu())
            ids = hs().clone()
            rids, _, _ = ref(h0)
            torch.cuda.synchronize()
            assert torch.equal(ids, rids.cpu())
        assert mq.device_error() == 0
    finally:
        hs.close()
