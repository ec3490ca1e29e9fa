"""GPU parity of the tcgen05 prefill GEMM (bf16 activations, more than 16 rows): Q4
quantized_matmul (src/model/marlin.cpp:18-25) and the fused SwiGLU / residual epilogues of
mlp_forward (:31-35).

The GEMM dequantizes each weight once into the activation type, bf16(s*q + b) with a single
rounding, as a quantized GEMM over many rows stages weight tiles, and accumulates in binary32.
References are float64 products with those weights (the path's tolerance, max relative error 1e-2
per row, plus a tight mean bound); single-rounding outputs are also held to the tolerance against
the exactly dequantized weights."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import TOL, act, host_q4, make_q4, max_rel_row_err

pytestmark = pytest.mark.gpu


def dequant(q: mq.QuantizedTensor) -> torch.Tensor:
    """Exact dequantization s*q + b (float64)."""
    h = host_q4(q)
    return torch.from_numpy(qo.np_dequant(h.weight, h.scales, h.biases)).cuda().double()


def dequant_bf16(deq: torch.Tensor) -> torch.Tensor:
    """The GEMM's operand: each exact s*q + b rounded once to bf16 (exact in binary32 first)."""
    return deq.float().to(torch.bfloat16).double()


def bf16r(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).double()


def swiglu_bf16_ref(gs: torch.Tensor, us: torch.Tensor) -> torch.Tensor:
    """swiglu (src/model/marlin.cpp:27-29) on bf16 tensors: every MLX op rounds its output to bf16."""
    gq, uq = bf16r(gs), bf16r(us)
    return bf16r(bf16r(bf16r(torch.sigmoid(gq)) * gq) * uq)


def mean_rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    den = ref.abs().amax(dim=1, keepdim=True).clamp_min(1e-30)
    return float(((y.double() - ref).abs() / den).mean())


@pytest.fixture(scope="module")
def mats():
    out = {}
    for i, (n, k) in enumerate([(6144, 2048), (2048, 6144), (1000, 512), (300, 1024), (6144, 2048)]):
        q, _ = make_q4(n, k, 900 + i)
        deq = dequant(q)
        out[i] = (q, deq, dequant_bf16(deq))
    return out


@pytest.mark.parametrize("idx,m", [(0, 17), (0, 300), (0, 2048), (0, 3900), (1, 129), (1, 2048), (2, 64),
                                   (2, 1000), (3, 33), (3, 257)])
def test_prefill_qmatmul(mats, idx, m):
    q, deq, deq16 = mats[idx]
    x = act((m, q.k), 10 + m, torch.bfloat16)
    y = mq.qmatmul(x, q)
    torch.cuda.synchronize()
    ref = x.double() @ deq16.T
    assert y.dtype == torch.bfloat16 and y.shape == (m, q.n)
    assert max_rel_row_err(y.float().cpu().numpy(), ref.cpu().numpy()) < TOL
    assert mean_rel_err(y, ref) < 1e-3
    exact = x.double() @ deq.T  # against the exactly dequantized weights, too
    assert max_rel_row_err(y.float().cpu().numpy(), exact.cpu().numpy()) < TOL
    assert mq.device_error() == 0


@pytest.mark.parametrize("m", [40, 300])
def test_prefill_gate_up_swiglu(mats, m):
    (g, _, dg), (u, _, du) = mats[0], mats[4]
    x = act((m, 2048), 30 + m, torch.bfloat16)
    a = mq.gate_up_swiglu(x, g, u)
    torch.cuda.synchronize()
    gs, us = x.double() @ dg.T, x.double() @ du.T
    ref = swiglu_bf16_ref(gs, us)
    assert a.dtype == torch.bfloat16 and a.shape == (m, 6144)
    assert max_rel_row_err(a.float().cpu().numpy(), ref.cpu().numpy()) < TOL
    assert mq.device_error() == 0


@pytest.mark.parametrize("resid_dtype", [torch.bfloat16, torch.float32])
def test_prefill_down_residual(mats, resid_dtype):
    d, _, dd = mats[1]
    m = 200
    a = act((m, 6144), 51, torch.bfloat16, sigma=0.1)
    h = act((m, 2048), 52, resid_dtype)
    y = mq.matmul_residual(a, d, h)
    torch.cuda.synchronize()
    delta = a.double() @ dd.T
    assert y.dtype == torch.float32
    assert max_rel_row_err((y.double() - h.double()).cpu().numpy(), delta.cpu().numpy()) < TOL
    assert mq.device_error() == 0


def test_prefill_c4_stack(mats):
    """Config 4: x bf16 [2048, 2048] through gate/up -> SwiGLU -> down at full size."""
    (g, _, dg), (u, _, du), (d, _, dd) = mats[0], mats[4], mats[1]
    x = act((2048, 2048), 77, torch.bfloat16)
    a = mq.gate_up_swiglu(x, g, u)
    y = mq.qmatmul(a, d)
    torch.cuda.synchronize()
    ref = a.double() @ dd.T  # the down GEMM against the produced activations
    assert max_rel_row_err(y.float().cpu().numpy(), ref.cpu().numpy()) < TOL
    gs, us = x.double() @ dg.T, x.double() @ du.T
    ref_a = swiglu_bf16_ref(gs, us)
    assert max_rel_row_err(a.float().cpu().numpy(), ref_a.cpu().numpy()) < TOL
    # deterministic: a second run gives identical bits
    y2 = mq.qmatmul(mq.gate_up_swiglu(x, g, u), d)
    assert torch.equal(y, y2)
    assert mq.device_error() == 0


@pytest.mark.parametrize("world", [2, 8])
def test_sharded_prefill_mlp_on_one_gpu(world):
    """The tensor-parallel prefill MLP's arithmetic with every shard run on this one GPU: each rank's
    gate/up rows (zero-padded to a multiple of 512 at 8 ranks, where a shard holds 768 rows) feed
    its binary32 down_proj partial (marlin_q4_matmul_f32, tcgen05 GEMM); the partials are summed in
    rank order and rounded once (marlin_q4_cast_bf16).  Against the single-GPU mlp_forward: within the
    path's tolerance and equal in nearly every element."""
    from marlin_q4 import tp
    S, H, I = 2048, 2048, 6144
    g, _ = make_q4(I, H, 601)
    u, _ = make_q4(I, H, 602)
    d, _ = make_q4(H, I, 603)
    layer = mq.Layer(mq.synth_bf16((H,), 604, 0.1, 0.02), g, u, d)
    x = mq.synth_bf16((S, H), 605, 0.0, 1.0)
    total = torch.zeros((S, H), dtype=torch.float32, device="cuda")
    for r in range(world):
        sh = tp.shard_layer(layer, r, world, k_multiple=512, pad_gate_up=True)
        assert sh.gate_proj.n == sh.down_proj.k and sh.down_proj.k % 512 == 0
        a = mq.gate_up_swiglu(x, sh.gate_proj, sh.up_proj)
        assert torch.count_nonzero(a[:, I // world:]) == 0  # the padded features are exact zeros
        total += mq.matmul_f32(a, sh.down_proj)
    y = mq.cast_bf16(total)
    ry = mq.mlp_forward(x, g, u, d)
    torch.cuda.synchronize()
    rel = ((y.float() - ry.float()).abs().amax(dim=1) / ry.float().abs().amax(dim=1)).max().item()
    assert rel < TOL
    assert (y.view(torch.int16) == ry.view(torch.int16)).float().mean().item() > 0.9
    assert torch.equal(mq.cast_bf16(ry.float()), ry)  # bf16 values survive the round trip
    assert mq.device_error() == 0
