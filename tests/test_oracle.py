"""CPU tests of the oracle: C restatement vs NumPy mirror vs golden vectors, and algebraic properties.

The oracle is the checker for the CUDA product; these tests pin it against its own independent
restatements and the hand-derived known-answer cases (MLX itself is absent: parity unpinned).
"""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

import q4_oracle as qo

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "q4_golden.npz")


def test_golden_manifest(golden):
    manifest = json.loads((GOLDEN / "q4_golden.sha256.json").read_text())
    assert sorted(manifest) == sorted(golden.files)
    for k in golden.files:
        assert hashlib.sha256(np.ascontiguousarray(golden[k]).tobytes()).hexdigest() == manifest[k], k


@pytest.mark.parametrize("seed,mean,sigma,key", [(1234, 0.0, 1.0, "synth_s1234_n01"), (7, 0.0, 0.02, "synth_s7_n002"),
                                                 (9, 0.1, 0.02, "synth_s9_n01_002")])
def test_generator_matches_golden(oracle, golden, seed, mean, sigma, key):
    assert np.array_equal(oracle.synth_bf16((4096,), seed, mean, sigma), golden[key])
    assert np.array_equal(qo.np_synth_bf16(4096, seed, mean, sigma), golden[key])


def test_generator_distribution(oracle):
    v = qo.bf16_to_f32(oracle.synth_bf16((1 << 20,), 5, 0.0, 1.0)).astype(np.float64)
    assert abs(v.mean()) < 5e-3 and abs(v.std() - 1.0) < 5e-3
    assert v.min() >= -6.0 and v.max() <= 6.0
    # offset stream start: element i of a stream does not depend on the buffer it is generated into
    assert np.array_equal(qo.np_synth_bf16(100, 5, 0.0, 1.0, start=1000),
                          oracle.synth_bf16((1100,), 5, 0.0, 1.0)[1000:])


def test_kat_hand_values(golden):
    from golden.make_golden import KAT_EXPECT
    for name, (words, s, b) in KAT_EXPECT.items():
        assert [int(x) for x in golden[f"kat_{name}_wq"][0]] == words
        assert int(golden[f"kat_{name}_s"][0, 0]) == s and int(golden[f"kat_{name}_b"][0, 0]) == b


@pytest.mark.parametrize("name", ["ramp_up", "ramp_down", "all_zero", "constant", "all_negative", "all_positive",
                                  "outlier", "tie", "param_order"])
def test_kat_c_oracle(oracle, golden, name):
    w = golden[f"kat_{name}_w"]
    q = oracle.quantize(w)
    assert np.array_equal(q.weight, golden[f"kat_{name}_wq"])
    assert np.array_equal(q.scales, golden[f"kat_{name}_s"])
    assert np.array_equal(q.biases, golden[f"kat_{name}_b"])
    for flags in (qo.ROUND_HALF_EVEN, qo.TRUE_MINMAX, qo.NO_ZERO_SNAP, qo.BF16_PARAMS_FIRST):
        q = oracle.quantize(w, flags)
        assert np.array_equal(q.weight, golden[f"kat_{name}_f{flags}_wq"])
        assert np.array_equal(q.scales, golden[f"kat_{name}_f{flags}_s"])


def test_kat_tie_rounding(golden):
    """Element 2 sits exactly on code 2.5: ties-away gives 3, ties-even gives 2."""
    codes_away = qo.np_unpack(golden["kat_tie_wq"])[0]
    codes_even = qo.np_unpack(golden["kat_tie_f1_wq"])[0]
    assert codes_away[2] == 3 and codes_even[2] == 2
    assert codes_away[3] == 4 and codes_even[3] == 4
    assert codes_away[4] == 1 and codes_even[4] == 0


def test_kat_param_order(golden):
    """The codes come from the binary32 scale and bias; only the stored copies are rounded to bf16.
    On this group the other order (bf16-rounded parameters first) moves elements 27 and 62 up by
    one code, while the stored scale and bias are the same either way."""
    first_f32 = qo.np_unpack(golden["kat_param_order_wq"])[0]
    first_bf16 = qo.np_unpack(golden["kat_param_order_f8_wq"])[0]
    assert list(np.nonzero(first_f32 != first_bf16)[0]) == [27, 62]
    assert list(first_f32[[27, 62]]) == [6, 10] and list(first_bf16[[27, 62]]) == [7, 11]
    assert np.array_equal(golden["kat_param_order_s"], golden["kat_param_order_f8_s"])
    assert np.array_equal(golden["kat_param_order_b"], golden["kat_param_order_f8_b"])


def test_quantize_error_bound():
    """Dequantized values stay within one quantization step of the input (half a step from rounding,
    up to one step at the far extreme that the edge snapping can push past code 15 and clamp)."""
    w = qo.np_synth_bf16(256 * 512, 77, 0.0, 0.02).reshape(256, 512)
    g = qo.bf16_to_f32(w).reshape(256, 8, 64)
    wmin, wmax = g.min(-1), np.maximum(g.max(-1), 0)
    assert np.all(wmin < 0) and np.all(wmax > 0)
    wq, s, b = qo.np_quantize(w)
    deq = qo.np_dequant(wq, s, b).reshape(256, 8, 64)
    step = np.abs(qo.bf16_to_f32(s))[..., None]
    err = np.abs(deq - g)
    assert np.all(err <= 1.05 * step + 1e-6)
    assert 0.2 < float((err / step).mean()) < 0.3


@pytest.mark.parametrize("flags", range(16))
def test_c_vs_numpy_quantize(oracle, golden, flags):
    w = golden["rand_q_w"]
    q = oracle.quantize(w, flags)
    wq, s, b = qo.np_quantize(w, flags)
    assert np.array_equal(q.weight, wq) and np.array_equal(q.scales, s) and np.array_equal(q.biases, b)
    if flags == 0:
        assert np.array_equal(q.weight, golden["rand_q_wq"])


def test_quantize_rejects_bad_shapes(oracle):
    w = np.zeros((4, 96), np.uint16)
    with pytest.raises(ValueError):
        oracle.quantize(w)
    with pytest.raises(ValueError):
        oracle.quantize(np.zeros((4, 64), np.uint16), group_size=32)
    with pytest.raises(ValueError):
        oracle.quantize(np.zeros((4, 64), np.uint16), bits=8)


def test_qmatmul_vs_f64(oracle, golden):
    w = golden["rand_q_w"]
    q = oracle.quantize(w)
    for key in ("f_qmm_xb", "f_qmm_xf"):
        x = golden[key]
        xf = qo.bf16_to_f32(x) if x.dtype == np.uint16 else x
        ref = qo.np_qmatmul_f64(xf, q.weight, q.scales, q.biases)
        y = oracle.qmatmul(x, q)
        err = np.abs(y - ref).max(axis=1) / np.abs(ref).max(axis=1)
        assert err.max() < 1e-5
    assert np.array_equal(oracle.qmatmul(golden["f_qmm_xb"], q), golden["f_qmm_yb"])
    assert np.array_equal(oracle.qmatmul(golden["f_qmm_xf"], q), golden["f_qmm_yf"])


def test_qmatmul_linearity(oracle):
    w = qo.np_synth_bf16(32 * 256, 3, 0.0, 0.02).reshape(32, 256)
    q = oracle.quantize(w)
    a = qo.bf16_to_f32(qo.np_synth_bf16(256, 4, 0.0, 1.0))[None]
    b = qo.bf16_to_f32(qo.np_synth_bf16(256, 5, 0.0, 1.0))[None]
    ya, yb, yab = oracle.qmatmul(a, q), oracle.qmatmul(b, q), oracle.qmatmul(a + b, q)
    assert np.allclose(ya + yb, yab, rtol=1e-5, atol=1e-5)


def test_rms_norm(oracle, golden):
    assert np.array_equal(oracle.rms_norm(golden["f_qmm_xb"], golden["f_norm_w"]), golden["f_norm_yb"])
    assert np.array_equal(oracle.rms_norm(golden["f_qmm_xf"], golden["f_norm_w"]), golden["f_norm_yf"])
    x = golden["f_qmm_xf"].astype(np.float64)
    w = qo.bf16_to_f32(golden["f_norm_w"]).astype(np.float64)
    ref = x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * (1 + w)
    assert np.allclose(golden["f_norm_yf"], ref, rtol=1e-5, atol=1e-6)


def test_swiglu(oracle, golden):
    g, u = golden["f_swiglu_g"].astype(np.float64), golden["f_swiglu_u"].astype(np.float64)
    ref = g / (1 + np.exp(-g)) * u
    assert np.allclose(oracle.swiglu_f32(golden["f_swiglu_g"], golden["f_swiglu_u"]), ref, rtol=1e-5, atol=1e-6)
    assert np.array_equal(oracle.swiglu_f32(golden["f_swiglu_g"], golden["f_swiglu_u"]), golden["f_swiglu_f32"])
    out = qo.bf16_to_f32(golden["f_swiglu_bf16"])
    assert np.allclose(out, ref, rtol=2e-2, atol=2e-2)


def _q(golden, p):
    return qo.Q4(golden[f"{p}_wq"], golden[f"{p}_s"], golden[f"{p}_b"])


def test_mlp(oracle, golden):
    gate, up, down = _q(golden, "f_mlp_gate"), _q(golden, "f_mlp_up"), _q(golden, "f_mlp_down")
    x = golden["f_mlp_x"]
    assert np.array_equal(oracle.mlp(x, gate, up, down), golden["f_mlp_yb"])
    assert np.array_equal(oracle.mlp(qo.bf16_to_f32(x), gate, up, down), golden["f_mlp_yf"])
    # f64 composition
    xf = qo.bf16_to_f32(x).astype(np.float64)
    G = xf @ qo.np_dequant(gate.weight, gate.scales, gate.biases).T
    U = xf @ qo.np_dequant(up.weight, up.scales, up.biases).T
    A = G / (1 + np.exp(-G)) * U
    Y = A @ qo.np_dequant(down.weight, down.scales, down.biases).T
    assert np.max(np.abs(golden["f_mlp_yf"] - Y)) / np.abs(Y).max() < 1e-5
    yb = qo.bf16_to_f32(golden["f_mlp_yb"])
    assert np.max(np.abs(yb - Y), axis=1).max() / np.abs(Y).max() < 1e-2


def test_argmax_first_index_on_ties(oracle):
    logits = np.array([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0], [-1.0, -0.5, -0.5, -2.0]], np.float32)
    ids = np.empty(3, np.int32)
    oracle.lib.q4o_argmax_f32(logits.ctypes.data, 3, 4, ids.ctypes.data, None)
    assert ids.tolist() == [1, 0, 1]


def test_lm_head_argmax(oracle, golden):
    lm = _q(golden, "f_lm")
    h = golden["f_lm_h"]
    ids, best = oracle.lm_head_argmax(h, lm)
    assert np.array_equal(ids, golden["f_lm_ids_bf16"]) and np.array_equal(best, golden["f_lm_best_bf16"])
    ids, best = oracle.lm_head_argmax(qo.bf16_to_f32(h), lm)
    assert np.array_equal(ids, golden["f_lm_ids_f32"])
    ref = qo.bf16_to_f32(h).astype(np.float64) @ qo.np_dequant(lm.weight, lm.scales, lm.biases).T.astype(np.float64)
    assert np.array_equal(ids, ref.argmax(axis=1).astype(np.int32))


def test_decode_step(oracle, golden):
    gate, up, down = _q(golden, "f_mlp_gate"), _q(golden, "f_mlp_up"), _q(golden, "f_mlp_down")
    lm = _q(golden, "f_lm")
    layers = [(golden["f_dec_norm0"], gate, up, down), (golden["f_dec_norm1"], up, gate, down)]
    ids, best, h = oracle.decode_step(golden["f_dec_h0"], layers, golden["f_dec_final"], lm)
    assert np.array_equal(ids, golden["f_dec_ids"]) and np.array_equal(h, golden["f_dec_h"])
    # the step equals its composition from the oracle's own operators
    hcur = golden["f_dec_h0"]
    h32 = qo.bf16_to_f32(hcur)
    for i, (nw, g, u, d) in enumerate(layers):
        p = oracle.rms_norm(hcur if i == 0 else h32, nw)
        h32 = h32 + oracle.mlp(p, g, u, d)
    assert np.array_equal(h32, h)
    ids2, _ = oracle.lm_head_argmax(oracle.rms_norm(h32, golden["f_dec_final"]), lm)
    assert np.array_equal(ids2, ids)


def test_thread_count_independence(oracle):
    """Results do not depend on the OpenMP thread count (fixed summation order)."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r); import q4_oracle as qo, numpy as np;"
            "C = qo.COracle(); w = C.synth_bf16((96, 512), 3, 0.0, 0.02); q = C.quantize(w);"
            "x = qo.bf16_to_f32(C.synth_bf16((2, 512), 4, 0.0, 1.0));"
            "print(qo.hashlib_digest(C.qmatmul(x, q)) if hasattr(qo, 'hashlib_digest') else "
            "__import__('hashlib').sha256(C.qmatmul(x, q).tobytes()).hexdigest())") % str(qo.HERE)
    outs = set()
    for t in ("1", "3", "8"):
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                           env={**__import__("os").environ, "OMP_NUM_THREADS": t}, check=True)
        outs.add(r.stdout.strip())
    assert len(outs) == 1
