"""GPU parity of the two decode kernel families — integer MMAs on the codes (default) and bf16
mma.sync — each against the CPU oracle and against each other on the same inputs."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import TOL, act, f32, host_act, host_q4, make_q4, max_rel_row_err, u16

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["i8", "bf16"])
def path(request):
    mq.set_decode_path(request.param)
    yield request.param
    mq.set_decode_path("i8")


@pytest.fixture(scope="module")
def mats():
    g, _ = make_q4(6144, 2048, 71)
    u, _ = make_q4(6144, 2048, 72)
    d, _ = make_q4(2048, 6144, 73)
    lm, _ = make_q4(40000, 2048, 74)
    nw = mq.synth_bf16((2048,), 75, 0.1, 0.02)
    return {"g": g, "u": u, "d": d, "lm": lm, "nw": nw,
            "hg": host_q4(g), "hu": host_q4(u), "hd": host_q4(d), "hlm": host_q4(lm), "hnw": u16(nw)}


@pytest.mark.parametrize("m,dtype", [(1, torch.float32), (1, torch.bfloat16), (2, torch.float32),
                                     (5, torch.float32), (7, torch.float32), (16, torch.bfloat16),
                                     (24, torch.bfloat16)])
def test_qmatmul_paths(oracle, mats, path, m, dtype):
    for q, hq, k in ((mats["g"], mats["hg"], 2048), (mats["d"], mats["hd"], 6144)):
        x = act((m, k), 80 + m, dtype)
        y = mq.qmatmul(x, q)
        ref = oracle.qmatmul(host_act(x), hq)
        if dtype == torch.bfloat16:
            assert max_rel_row_err(qo.bf16_to_f32(u16(y)), ref) < TOL
            # above 16 rows bf16 inputs take the prefill GEMM (weights dequantized to bf16)
            assert np.mean(u16(y) == qo.f32_to_bf16(ref)) > (0.99 if m <= 16 else 0.5)
        else:
            assert max_rel_row_err(f32(y), ref) < 2e-5
    assert mq.device_error() == 0


@pytest.mark.parametrize("m", [1, 3])
def test_fused_layer_paths(oracle, mats, path, m):
    h = act((m, 2048), 90 + m, torch.float32)
    a = mq.gate_up_swiglu(h, mats["g"], mats["u"], norm_weight=mats["nw"])
    p = oracle.rms_norm(host_act(h), mats["hnw"])
    ref_a = oracle.swiglu_f32(oracle.qmatmul(p, mats["hg"]), oracle.qmatmul(p, mats["hu"]))
    assert max_rel_row_err(f32(a), ref_a) < 1e-4
    y = mq.matmul_residual(a, mats["d"], h)
    ref_y = host_act(h) + oracle.qmatmul(f32(a), mats["hd"])
    assert max_rel_row_err(f32(y), ref_y) < 1e-5
    assert mq.device_error() == 0


@pytest.mark.parametrize("m,dtype,norm", [(1, torch.bfloat16, True), (4, torch.bfloat16, True),
                                          (1, torch.float32, False), (3, torch.bfloat16, False),
                                          (16, torch.bfloat16, False)])
def test_lm_head_paths(oracle, mats, path, m, dtype, norm):
    h = act((m, 2048), 100 + m, dtype)
    nw = mats["nw"] if norm else None
    ids, best = mq.lm_head_argmax(h, mats["lm"], norm_weight=nw)
    hx = oracle.rms_norm(host_act(h), mats["hnw"]) if norm else host_act(h)
    rids, rbest = oracle.lm_head_argmax(hx, mats["hlm"])
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert mq.device_error() == 0


def test_paths_agree_on_decode_layer(mats):
    h = act((2, 2048), 110, torch.float32)
    outs = []
    for p in ("i8", "bf16"):
        mq.set_decode_path(p)
        a = mq.gate_up_swiglu(h, mats["g"], mats["u"], norm_weight=mats["nw"])
        outs.append(f32(mq.matmul_residual(a, mats["d"], h)))
    mq.set_decode_path("i8")
    for o in outs[1:]:
        assert max_rel_row_err(outs[0], o.astype(np.float64)) < 1e-5
