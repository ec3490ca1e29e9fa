"""Generate tests/golden/q4_golden.npz — the oracle's golden vectors.

    python tests/golden/make_golden.py

Contents
  * kat_*      hand-derivable quantize known-answer cases (inputs exact in bf16; expected words,
               scales and biases are written out literally below and checked against the oracle);
  * synth_*    generator output for fixed seeds (NumPy mirror of the seeded generator);
  * rand_q_*   seeded random quantize case (NumPy mirror);
  * f_*        float-path regression vectors produced by the C oracle (qmatmul, rms_norm, swiglu,
               mlp in both dtype flows, lm_head argmax, a two-layer decode step).

The reference ships no tests or golden vectors and MLX (which owns the arithmetic) is absent here,
so these vectors pin the restatement against itself (C vs NumPy mirror, and over time); they do not
pin it to MLX: parity is unpinned.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "oracle"))
import q4_oracle as qo  # noqa: E402

OUT = HERE / "q4_golden.npz"


def bf(vals) -> np.ndarray:
    return qo.f32_to_bf16(np.asarray(vals, dtype=np.float32))


def kat_inputs() -> dict[str, np.ndarray]:
    j = np.arange(64)
    tie = np.full(64, -0.5, np.float32)
    tie[1] = 0.4375                       # max; range 0.9375 -> s = 0.0625, q0 = -8, b = -0.5
    tie[2] = -0.5 + 2.5 * 0.0625          # code 2.5: ties away -> 3, ties even -> 2
    tie[3] = -0.5 + 3.5 * 0.0625          # 3.5 -> 4 either way
    tie[4] = -0.5 + 0.5 * 0.0625          # 0.5: away -> 1, even -> 0
    tie[5:] = -0.5 + (j[5:] % 15) * 0.0625
    outlier = np.where(j % 2 == 0, 0.01, -0.01).astype(np.float32)
    outlier[17] = 1.0
    return {
        "ramp_up": bf([[(i % 16) * 0.125 - 1.0 for i in range(64)]]),
        "ramp_down": bf([[1.625 - (i % 16) * 0.125 for i in range(64)]]),
        "all_zero": bf(np.zeros((1, 64))),
        "constant": bf(np.full((1, 64), 0.5)),
        "all_negative": bf([[-0.25 - (i % 13) * 0.0625 for i in range(64)]]),
        "all_positive": bf([[0.25 + (i % 13) * 0.0625 for i in range(64)]]),
        "outlier": bf(outlier[None, :]),
        "tie": bf(tie[None, :]),
        # a seeded group whose codes at elements 27 and 62 depend on the order of the roundings:
        # codes from the binary32 scale and bias give 6 and 10; from the bf16-rounded ones, 7 and 11
        "param_order": qo.np_synth_bf16(64, 100, 0.0, 0.02).reshape(1, 64),
    }


# Hand-derived expectations (MLX affine quantize with zero snapping, round half away from zero).
KAT_EXPECT = {
    # s = 1.875/15 = 0.125, |min| > max -> edge = -1, q0 = -8, s = 0.125, b = -1, q = j % 16
    "ramp_up": ([0x76543210, 0xFEDCBA98] * 4, 0x3E00, 0xBF80),
    # |min| = 0.25 < max = 1.625 -> s = -0.125, edge = 1.625, q0 = -13, b = 1.625, q = j % 16
    "ramp_down": ([0x76543210, 0xFEDCBA98] * 4, 0xBE00, 0x3FD0),
    # max = min = 0 -> s = -1e-7, q0 = -0 == 0 -> b = 0, all codes 0
    "all_zero": ([0] * 8, 0xB3D7, 0x0000),
}


def main() -> None:
    C = qo.COracle()
    data: dict[str, np.ndarray] = {}

    for name, w in kat_inputs().items():
        data[f"kat_{name}_w"] = w
        wq, s, b = qo.np_quantize(w)
        data[f"kat_{name}_wq"], data[f"kat_{name}_s"], data[f"kat_{name}_b"] = wq, s, b
        for flags in (qo.ROUND_HALF_EVEN, qo.TRUE_MINMAX, qo.NO_ZERO_SNAP, qo.BF16_PARAMS_FIRST):
            wq2, s2, b2 = qo.np_quantize(w, flags)
            data[f"kat_{name}_f{flags}_wq"], data[f"kat_{name}_f{flags}_s"], data[f"kat_{name}_f{flags}_b"] = wq2, s2, b2
    for name, (words, s, b) in KAT_EXPECT.items():
        assert [int(v) for v in data[f"kat_{name}_wq"][0]] == words, name
        assert int(data[f"kat_{name}_s"][0, 0]) == s and int(data[f"kat_{name}_b"][0, 0]) == b, name

    data["synth_s1234_n01"] = qo.np_synth_bf16(4096, 1234, 0.0, 1.0)
    data["synth_s7_n002"] = qo.np_synth_bf16(4096, 7, 0.0, 0.02)
    data["synth_s9_n01_002"] = qo.np_synth_bf16(4096, 9, 0.1, 0.02)

    w = qo.np_synth_bf16(64 * 512, 11, 0.0, 0.02).reshape(64, 512)
    data["rand_q_w"] = w
    data["rand_q_wq"], data["rand_q_s"], data["rand_q_b"] = qo.np_quantize(w)

    # float-path regression vectors from the C oracle
    M, K, N = 3, 512, 64
    q = C.quantize(w)
    xb = qo.np_synth_bf16(M * K, 21, 0.0, 1.0).reshape(M, K)
    xf = qo.bf16_to_f32(qo.np_synth_bf16(M * K, 22, 0.0, 1.0).reshape(M, K)) * np.float32(1.25)
    data["f_qmm_xb"], data["f_qmm_xf"] = xb, xf
    data["f_qmm_yb"] = C.qmatmul(xb, q)
    data["f_qmm_yf"] = C.qmatmul(xf, q)
    nw = qo.np_synth_bf16(K, 23, 0.1, 0.02)
    data["f_norm_w"] = nw
    data["f_norm_yb"] = C.rms_norm(xb, nw)
    data["f_norm_yf"] = C.rms_norm(xf, nw)
    g = qo.bf16_to_f32(qo.np_synth_bf16(256, 24, 0.0, 2.0))
    u = qo.bf16_to_f32(qo.np_synth_bf16(256, 25, 0.0, 2.0))
    data["f_swiglu_g"], data["f_swiglu_u"] = g, u
    data["f_swiglu_f32"] = C.swiglu_f32(g, u)
    data["f_swiglu_bf16"] = C.swiglu_bf16(qo.f32_to_bf16(g), qo.f32_to_bf16(u))

    H, I = 128, 256
    gate = C.quantize(qo.np_synth_bf16(I * H, 31, 0.0, 0.02).reshape(I, H))
    up = C.quantize(qo.np_synth_bf16(I * H, 32, 0.0, 0.02).reshape(I, H))
    down = C.quantize(qo.np_synth_bf16(H * I, 33, 0.0, 0.02).reshape(H, I))
    for nm, t in (("gate", gate), ("up", up), ("down", down)):
        data[f"f_mlp_{nm}_wq"], data[f"f_mlp_{nm}_s"], data[f"f_mlp_{nm}_b"] = t.weight, t.scales, t.biases
    hx = qo.np_synth_bf16(2 * H, 34, 0.0, 1.0).reshape(2, H)
    data["f_mlp_x"] = hx
    data["f_mlp_yb"] = C.mlp(hx, gate, up, down)
    data["f_mlp_yf"] = C.mlp(qo.bf16_to_f32(hx), gate, up, down)

    V = 1000
    lm = C.quantize(qo.np_synth_bf16(V * H, 41, 0.0, 0.02).reshape(V, H))
    data["f_lm_wq"], data["f_lm_s"], data["f_lm_b"] = lm.weight, lm.scales, lm.biases
    hid = qo.np_synth_bf16(4 * H, 42, 0.0, 1.0).reshape(4, H)
    data["f_lm_h"] = hid
    ids, best = C.lm_head_argmax(hid, lm)
    data["f_lm_ids_bf16"], data["f_lm_best_bf16"] = ids, best
    ids, best = C.lm_head_argmax(qo.bf16_to_f32(hid), lm)
    data["f_lm_ids_f32"], data["f_lm_best_f32"] = ids, best

    norms = [qo.np_synth_bf16(H, 50 + l, 0.1, 0.02) for l in range(2)]
    layers = [(norms[0], gate, up, down), (norms[1], up, gate, down)]
    fn = qo.np_synth_bf16(H, 60, 0.1, 0.02)
    h0 = qo.np_synth_bf16(2 * H, 61, 0.0, 1.0).reshape(2, H)
    data["f_dec_norm0"], data["f_dec_norm1"], data["f_dec_final"], data["f_dec_h0"] = norms[0], norms[1], fn, h0
    ids, best, h = C.decode_step(h0, layers, fn, lm)
    data["f_dec_ids"], data["f_dec_best"], data["f_dec_h"] = ids, best, h

    np.savez_compressed(OUT, **data)
    manifest = {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest() for k, v in sorted(data.items())}
    (HERE / "q4_golden.sha256.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    main()
