"""GPU parity of the same Q4 operator at the shapes of the reference's other linear layers, the next
call sites for Q4 weights (the mixer projections that carry the next ~25 % of decode bytes):

  gated DeltaNet (src/model/gated_deltanet.cpp:108-111, :183, :210; 16 key and 16 value heads of
  128, src/core/config.h:28-31): in_proj_qkv [6144, 2048], in_proj_z [2048, 2048], in_proj_a and
  in_proj_b [16, 2048], out_proj [2048, 2048];
  full attention (src/model/attention.cpp:82-89, :139; 8 query heads of 256 with a gate, 2 KV heads,
  config.h:16-18): q_proj [4096, 2048], k_proj / v_proj [512, 2048], o_proj [2048, 2048].

marlin_q4_matmul takes any n and any k % 64 == 0, so these need no new kernel: decode rows go through
the integer-MMA GEMV family, prefill rows through the tcgen05 GEMM.  Checked against the CPU oracle
with the path's tolerance (max relative error 1e-2 per row)."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import TOL, act, host_act, host_q4, make_q4, max_rel_row_err, u16

pytestmark = pytest.mark.gpu

PROJ = {
    "deltanet.in_proj_qkv": (6144, 2048),
    "deltanet.in_proj_z": (2048, 2048),
    "deltanet.in_proj_b": (16, 2048),
    "deltanet.out_proj": (2048, 2048),
    "attn.q_proj": (4096, 2048),
    "attn.k_proj": (512, 2048),
}


@pytest.fixture(scope="module")
def mats():
    return {name: (lambda q: (q, host_q4(q)))(make_q4(n, k, 1300 + i)[0]) for i, (name, (n, k)) in enumerate(PROJ.items())}


@pytest.mark.parametrize("name", list(PROJ))
@pytest.mark.parametrize("m", [1, 4, 300])
def test_projection_shapes(oracle, mats, name, m):
    q, hq = mats[name]
    x = act((m, q.k), 1400 + m, torch.bfloat16)
    y = mq.qmatmul(x, q)
    torch.cuda.synchronize()
    ref = oracle.qmatmul(host_act(x), hq)
    assert y.shape == (m, q.n)
    assert max_rel_row_err(qo.bf16_to_f32(u16(y)), ref) < TOL
    if m <= 16:  # decode rows keep every product exact: nearly all outputs equal the oracle's rounding
        assert np.mean(u16(y) == qo.f32_to_bf16(ref)) > 0.99
    assert mq.device_error() == 0
