"""GPU parity: Q4 quantized_matmul (transpose=true, gs 64) against the CPU oracle.

bf16 activations -> bf16 output: within the path's tolerance (max rel error 1e-2 vs the fp32-
accumulated reference) and, for decode-sized m (<= 16), equal to the oracle's bf16 rounding for
nearly every element.  Above 16 rows bf16 inputs take the tcgen05 prefill GEMM, which rounds the
dequantized weights to bf16 (as a bf16 tensor-core operand must be), so there only the tolerance
and a majority of identical bf16 outputs are required.
binary32 activations -> binary32 output: the kernel splits x exactly into three bf16 planes, so it
must agree with the fp32 oracle to accumulation-order noise (max rel row error 2e-5)."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import TOL, act, f32, host_act, host_q4, make_q4, max_rel_row_err, u16

pytestmark = pytest.mark.gpu

SHAPES = [(6144, 2048), (2048, 6144), (100, 64), (7, 192), (1003, 512), (17, 128)]


@pytest.fixture(scope="module")
def weights():
    out = {}
    for i, (n, k) in enumerate(SHAPES):
        q, _ = make_q4(n, k, 500 + i)
        out[(n, k)] = (q, host_q4(q))
    return out


def _check(oracle, x, q, hq):
    y = mq.qmatmul(x, q)
    torch.cuda.synchronize()
    ref = oracle.qmatmul(host_act(x), hq)
    if x.dtype == torch.bfloat16:
        yb = u16(y)
        assert max_rel_row_err(qo.bf16_to_f32(yb), ref) < TOL
        same = np.mean(yb == qo.f32_to_bf16(ref))
        assert same > (0.99 if x.reshape(-1, x.shape[-1]).shape[0] <= 16 else 0.5), same
    else:
        assert max_rel_row_err(f32(y), ref) < 2e-5
    assert mq.device_error() == 0


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_qmatmul_decode_rows(oracle, weights, shape, dtype):
    q, hq = weights[shape]
    for m in (1, 2, 3, 5):
        _check(oracle, act((m, shape[1]), 7 + m, dtype), q, hq)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("m", [4, 8, 10, 11, 16, 17, 32, 33])
def test_qmatmul_batch_rows(oracle, weights, dtype, m):
    for shape in ((6144, 2048), (2048, 6144), (1003, 512)):
        q, hq = weights[shape]
        _check(oracle, act((m, shape[1]), 40 + m, dtype), q, hq)


def test_qmatmul_3d_input_and_linearity(oracle, weights):
    q, hq = weights[(6144, 2048)]
    a = act((1, 1, 2048), 1, torch.float32)
    b = act((1, 1, 2048), 2, torch.float32)
    ya, yb, yab = mq.qmatmul(a, q), mq.qmatmul(b, q), mq.qmatmul(a + b, q)
    assert ya.shape == (1, 1, 6144)
    assert torch.allclose(ya + yb, yab, rtol=1e-4, atol=1e-4)


def test_qmatmul_matches_dense_dequant(weights):
    """Independent check against torch: x @ dequant(W)^T in float64 on the GPU."""
    q, hq = weights[(2048, 6144)]
    deq = torch.from_numpy(qo.np_dequant(hq.weight, hq.scales, hq.biases)).cuda().double()
    x = act((3, 6144), 9, torch.float32)
    ref = (x.double() @ deq.T).cpu().numpy()
    assert max_rel_row_err(f32(mq.qmatmul(x, q)), ref) < 2e-5


def test_qmatmul_without_pdl(oracle, weights):
    q, hq = weights[(1003, 512)]
    mq.set_pdl(False)
    try:
        _check(oracle, act((2, 512), 3, torch.bfloat16), q, hq)
    finally:
        mq.set_pdl(True)
