"""GPU parity: the SwiGLU MLP block (src/model/marlin.cpp:27-35), RMSNorm (:12-16), and the fused
decode-layer kernels, against the CPU oracle."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import TOL, act, f32, host_act, host_q4, make_q4, max_rel_row_err, u16

pytestmark = pytest.mark.gpu

H, I = 2048, 6144


@pytest.fixture(scope="module")
def mlp():
    gate, _ = make_q4(I, H, 11)
    up, _ = make_q4(I, H, 12)
    down, _ = make_q4(H, I, 13)
    norm = mq.synth_bf16((H,), 14, 0.1, 0.02)
    return gate, up, down, norm, host_q4(gate), host_q4(up), host_q4(down), u16(norm)


@pytest.mark.parametrize("m", [1, 4, 16])
def test_mlp_bf16_config2(oracle, mlp, m):
    """Config 2: x bf16 [M,2048] ~N(0,1), gate/up/down Q4, out = down(silu(gate x) * up x)."""
    gate, up, down, _, hg, hu, hd, _ = mlp
    x = act((m, H), 20 + m, torch.bfloat16)
    y = mq.mlp_forward(x, gate, up, down)
    ref_b = oracle.mlp(u16(x), hg, hu, hd)
    xf = qo.bf16_to_f32(u16(x))
    ref32 = oracle.mlp(xf, hg, hu, hd)  # fp32-accumulated dequant reference
    assert y.dtype == torch.bfloat16
    # the oracle rounds to bf16 at the reference's op boundaries (gate, up, SwiGLU, out)
    assert max_rel_row_err(qo.bf16_to_f32(u16(y)), qo.bf16_to_f32(ref_b)) < TOL
    # and the bf16 flow stays close to the all-binary32 evaluation
    assert max_rel_row_err(qo.bf16_to_f32(u16(y)), ref32) < 5e-2


@pytest.mark.parametrize("m", [1, 3, 8, 10, 12])
def test_mlp_f32(oracle, mlp, m):
    gate, up, down, _, hg, hu, hd, _ = mlp
    x = act((m, H), 30 + m, torch.float32)
    y = mq.mlp_forward(x, gate, up, down)
    assert y.dtype == torch.float32
    assert max_rel_row_err(f32(y), oracle.mlp(host_act(x), hg, hu, hd)) < 1e-4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rms_norm(oracle, mlp, dtype):
    norm, hn = mlp[3], mlp[7]
    x = act((5, H), 40, dtype)
    y = f32(mq.rms_norm(x, norm))
    ref = oracle.rms_norm(host_act(x), hn)
    assert np.max(np.abs(y - ref) / np.maximum(np.abs(ref), 1e-3)) < 1e-5


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("m", [1, 8])
def test_fused_norm_gate_up_swiglu(oracle, mlp, dtype, m):
    gate, up, _, norm, hg, hu, _, hn = mlp
    x = act((m, H), 50 + m, dtype)
    a = mq.gate_up_swiglu(x, gate, up, norm_weight=norm)
    p = oracle.rms_norm(host_act(x), hn)
    g = oracle.qmatmul(p, hg)
    u = oracle.qmatmul(p, hu)
    ref = oracle.swiglu_f32(g, u)
    assert a.dtype == torch.float32
    assert max_rel_row_err(f32(a), ref) < 1e-4


@pytest.mark.parametrize("resid_dtype", [torch.bfloat16, torch.float32])
def test_down_residual(oracle, mlp, resid_dtype):
    _, _, down, _, _, _, hd, _ = mlp
    a = act((3, I), 60, torch.float32) * 0.1
    r = act((3, H), 61, resid_dtype)
    y = mq.matmul_residual(a, down, r)
    ref = host_act(r).astype(np.float32) if resid_dtype == torch.float32 else qo.bf16_to_f32(u16(r))
    ref = ref + oracle.qmatmul(host_act(a), hd)
    assert max_rel_row_err(f32(y), ref) < 1e-5
    # in place on a binary32 residual stream
    if resid_dtype == torch.float32:
        r2 = r.clone()
        mq.matmul_residual(a, down, r2, out=r2)
        assert torch.equal(r2, y)


def test_residual_add(mlp):
    h = act((2, H), 70, torch.bfloat16)
    y = act((2, H), 71, torch.float32)
    out = mq.residual_add(h, y)
    assert torch.equal(out, h.float() + y)
