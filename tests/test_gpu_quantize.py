"""GPU parity: seeded generator and Q4 quantize/pack are bit-exact against the CPU oracle."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import from_u16, u16, u32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,seed,mean,sigma", [(1, 1, 0.0, 1.0), (4097, 2, 0.0, 0.02), (10_000_019, 3, 0.1, 0.02)])
def test_synth_matches_oracle(oracle, n, seed, mean, sigma):
    g = u16(mq.synth_bf16((n,), seed, mean, sigma))
    assert np.array_equal(g, oracle.synth_bf16((n,), seed, mean, sigma))


@pytest.mark.parametrize("n,k", [(1, 64), (7, 128), (64, 512), (33, 192), (6144, 2048), (2048, 6144)])
def test_quantize_bit_exact(oracle, n, k):
    q, w = None, mq.synth_bf16((n, k), 100 + n + k, 0.0, 0.02)
    q = mq.quantize_weight(w)
    ref = oracle.quantize(u16(w))
    assert np.array_equal(u32(q.weight), ref.weight)
    assert np.array_equal(u16(q.scales), ref.scales)
    assert np.array_equal(u16(q.biases), ref.biases)


def test_quantize_lm_head_size(oracle):
    """The tied lm_head shape [248320, 2048] (src/model/weights.cpp:183)."""
    w = mq.synth_bf16((248320, 2048), 7, 0.0, 0.02)
    q = mq.quantize_weight(w)
    ref = oracle.quantize(u16(w))
    assert np.array_equal(u32(q.weight), ref.weight)
    assert np.array_equal(u16(q.scales), ref.scales) and np.array_equal(u16(q.biases), ref.biases)


def test_quantize_known_answers():
    from pathlib import Path
    g = np.load(Path(__file__).resolve().parent / "golden" / "q4_golden.npz")
    for name in ("ramp_up", "ramp_down", "all_zero", "constant", "all_negative", "all_positive", "outlier", "tie",
                 "param_order"):
        q = mq.quantize_weight(from_u16(g[f"kat_{name}_w"]))
        assert np.array_equal(u32(q.weight), g[f"kat_{name}_wq"]), name
        assert np.array_equal(u16(q.scales), g[f"kat_{name}_s"]), name
        assert np.array_equal(u16(q.biases), g[f"kat_{name}_b"]), name


def test_quantize_special_values(oracle):
    """Subnormal-scale groups, huge magnitudes and exact zeros mixed in one matrix."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((16, 256)).astype(np.float32) * 0.02
    w[0] = 0.0
    w[1] *= 1e-30
    w[2] *= 1e30
    w[3, ::2] = 0.0
    wb = qo.f32_to_bf16(w)
    q = mq.quantize_weight(from_u16(wb))
    ref = oracle.quantize(wb)
    assert np.array_equal(u32(q.weight), ref.weight)
    assert np.array_equal(u16(q.scales), ref.scales) and np.array_equal(u16(q.biases), ref.biases)


def test_quantize_rejects_bad_shape():
    with pytest.raises(mq.MarlinQ4Error):
        mq.quantize_weight(torch.zeros((8, 96), dtype=torch.bfloat16, device="cuda"))
