"""The on-disk Q4 weight cache (marlin_q4.cache): safetensors layout with MLX's quantized names
(name.weight U32 [n, k/8], name.scales / name.biases BF16 [n, k/64]), read back bit for bit.
CPU tests check the file format with an independent reader; the GPU test runs the decode step on
weights loaded from the cache against the same weights never written."""
import json
import struct

import numpy as np
import pytest
import torch

import marlin_q4 as mq
from marlin_q4 import cache


def rand_q4(n: int, k: int, seed: int) -> mq.QuantizedTensor:
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-2**31, 2**31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
    s = torch.randint(0, 2**16, (n, k // 64), generator=g, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    b = torch.randint(0, 2**16, (n, k // 64), generator=g, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    return mq.QuantizedTensor(w, s, b)


def same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype == torch.bfloat16:
        a, b = a.view(torch.int16), b.view(torch.int16)
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.cpu(), b.cpu())


def test_round_trip_bit_exact(tmp_path):
    q = {"a.proj": rand_q4(5, 128, 1), "lm_head": rand_q4(3, 64, 2)}
    plain = {"norm.weight": torch.randn(128).to(torch.bfloat16), "x.f32": torch.randn(3, 4)}
    path = tmp_path / "c.safetensors"
    cache.save(path, q, plain, {"note": "test"})
    q2, p2, meta = cache.load(path, device="cpu")
    assert set(q2) == set(q) and set(p2) == set(plain)
    for k in q:
        assert same_bits(q[k].weight, q2[k].weight) and same_bits(q[k].scales, q2[k].scales)
        assert same_bits(q[k].biases, q2[k].biases) and q2[k].group_size == 64 and q2[k].bits == 4
    for k in plain:
        assert same_bits(plain[k], p2[k])
    assert meta["note"] == "test" and meta["group_size"] == "64" and meta["bits"] == "4"


def test_file_layout_independent_reader(tmp_path):
    q = rand_q4(7, 192, 3)
    path = tmp_path / "one.safetensors"
    cache.save(path, {"w": q})
    raw = path.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    want = {"w.weight": ("U32", [7, 24], q.weight.numpy().view(np.uint32)),
            "w.scales": ("BF16", [7, 3], q.scales.view(torch.int16).numpy().view(np.uint16)),
            "w.biases": ("BF16", [7, 3], q.biases.view(torch.int16).numpy().view(np.uint16))}
    assert set(header) == set(want) | {"__metadata__"}
    for name, (dt, shape, arr) in want.items():
        h = header[name]
        assert h["dtype"] == dt and h["shape"] == shape
        b0, b1 = h["data_offsets"]
        assert b0 % 8 == 0 and b1 - b0 == arr.nbytes
        assert data[b0:b1] == arr.tobytes()  # row-major, little-endian, untouched


def test_model_names_follow_the_reference(tmp_path):
    layers = [mq.Layer(torch.randn(64).to(torch.bfloat16), rand_q4(128, 64, 10 + i), rand_q4(128, 64, 20 + i),
                       rand_q4(64, 128, 30 + i)) for i in range(2)]
    fn, lm = torch.randn(64).to(torch.bfloat16), rand_q4(256, 64, 40)
    path = tmp_path / "m.safetensors"
    cache.save_model(path, layers, fn, lm)
    header, _ = cache.read_header(path)
    for name in ("model.language_model.layers.1.mlp.down_proj.weight",
                 "model.language_model.layers.0.mlp.gate_proj.scales",
                 "model.language_model.layers.1.post_attention_layernorm.weight",
                 "model.language_model.norm.weight", "lm_head.weight", "lm_head.biases"):
        assert name in header
    l2, fn2, lm2 = cache.load_model(path, device="cpu")
    assert len(l2) == 2 and same_bits(fn2, fn) and same_bits(lm2.weight, lm.weight)
    for a, b in zip(layers, l2):
        for f in ("gate_proj", "up_proj", "down_proj"):
            assert same_bits(getattr(a, f).weight, getattr(b, f).weight)
            assert same_bits(getattr(a, f).scales, getattr(b, f).scales)
        assert same_bits(a.post_attn_norm, b.post_attn_norm)


@pytest.mark.gpu
def test_decode_step_from_cache_matches(tmp_path):
    H, I, V = 512, 1024, 2048
    layers = []
    for l in range(2):
        layers.append(mq.Layer(mq.synth_bf16((H,), 903 + 4 * l, 0.1, 0.02),
                               mq.quantize_weight(mq.synth_bf16((I, H), 900 + 4 * l, 0.0, 0.02)),
                               mq.quantize_weight(mq.synth_bf16((I, H), 901 + 4 * l, 0.0, 0.02)),
                               mq.quantize_weight(mq.synth_bf16((H, I), 902 + 4 * l, 0.0, 0.02))))
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 950, 0.0, 0.02))
    fn = mq.synth_bf16((H,), 951, 0.1, 0.02)
    path = tmp_path / "q4.safetensors"
    cache.save_model(path, layers, fn, lm)
    l2, fn2, lm2 = cache.load_model(path)
    h0 = mq.synth_bf16((2, H), 952, 0.0, 1.0)
    ids, _, h = (t.clone() for t in mq.DecodeStep(layers, fn, lm, 2)(h0))
    ids2, _, h2 = mq.DecodeStep(l2, fn2, lm2, 2)(h0)
    torch.cuda.synchronize()
    assert torch.equal(ids, ids2) and torch.equal(h, h2)
    assert mq.device_error() == 0
