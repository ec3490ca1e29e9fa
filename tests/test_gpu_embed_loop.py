"""GPU parity of the pieces around the decode step: the embedding rows from the tied Q4 table
(marlin_q4_embed; MarlinModel::embed_tokens, src/model/marlin.cpp:63-65, served from the quantized
lm_head), the greedy loop that feeds each step's ids back through it on the device
(marlin_q4.GreedyLoop; run_decode_loop, src/core/engine.cpp:79-94), and the token that starts the
loop after a prefill, from the last row only (src/core/engine.cpp:64 with sampler.cpp:10-15)."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import host_q4, make_q4, u16

pytestmark = pytest.mark.gpu


def dequant_rows_bf16(hq: qo.Q4, ids: np.ndarray) -> np.ndarray:
    """bf16 bits of s*q + b for rows `ids`, the exact value (float64) rounded once to bf16."""
    q = qo.np_unpack(hq.weight[ids]).astype(np.float64)
    s = np.repeat(qo.bf16_to_f32(hq.scales[ids]).astype(np.float64), qo.GROUP, axis=1)
    b = np.repeat(qo.bf16_to_f32(hq.biases[ids]).astype(np.float64), qo.GROUP, axis=1)
    exact = s * q + b
    f = exact.astype(np.float32)
    assert np.array_equal(f.astype(np.float64), exact)  # exact in binary32, so one bf16 rounding follows
    return qo.f32_to_bf16(f)


def test_embed_rows_bit_exact():
    V, H = 3000, 512
    lm, _ = make_q4(V, H, 700)
    rng = np.random.default_rng(5)
    ids_np = np.concatenate([[0, V - 1, 17, 17], rng.integers(0, V, 33)]).astype(np.int32)
    ids = torch.from_numpy(ids_np).cuda()
    out = mq.embed_q4(ids, lm)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == (ids_np.size, H)
    assert np.array_equal(u16(out), dequant_rows_bf16(host_q4(lm), ids_np))
    assert mq.device_error() == 0


def test_embed_out_of_range_ids_give_zero_rows_and_error():
    V, H = 256, 128
    lm, _ = make_q4(V, H, 701)
    ids = torch.tensor([3, -1, V, 5], dtype=torch.int32, device="cuda")
    out = mq.embed_q4(ids, lm)
    torch.cuda.synchronize()
    assert mq.device_error() == 3  # recorded (and cleared) by the kernel's bounds check
    o = u16(out)
    assert not o[1].any() and not o[2].any()
    assert np.array_equal(o[[0, 3]], dequant_rows_bf16(host_q4(lm), np.array([3, 5])))
    assert mq.device_error() == 0


def test_greedy_loop_matches_oracle(oracle):
    H, I, V, NL, m, T = 512, 1024, 2048, 2, 2, 4
    layers, host_layers = [], []
    for l in range(NL):
        g, _ = make_q4(I, H, 800 + 4 * l)
        u, _ = make_q4(I, H, 801 + 4 * l)
        d, _ = make_q4(H, I, 802 + 4 * l)
        nw = mq.synth_bf16((H,), 803 + 4 * l, 0.1, 0.02)
        layers.append(mq.Layer(nw, g, u, d))
        host_layers.append((u16(nw), host_q4(g), host_q4(u), host_q4(d)))
    lm, _ = make_q4(V, H, 850)
    fn = mq.synth_bf16((H,), 851, 0.1, 0.02)
    hlm = host_q4(lm)
    ids0 = np.array([7, 1500], dtype=np.int32)
    loop = mq.GreedyLoop(layers, fn, lm, m)
    got = loop(torch.from_numpy(ids0).cuda(), T)
    torch.cuda.synchronize()
    want, cur = [], ids0
    for _ in range(T):
        rids, _, _ = oracle.decode_step(dequant_rows_bf16(hlm, cur), host_layers, u16(fn), hlm)
        want.append(rids)
        cur = rids.astype(np.int32)
    assert np.array_equal(got.cpu().numpy(), np.stack(want))
    assert mq.device_error() == 0


def test_next_token_after_prefill_is_last_row_argmax():
    S, H, V = 40, 512, 2048
    lm, _ = make_q4(V, H, 860)
    fn = mq.synth_bf16((H,), 861, 0.1, 0.02)
    hidden = mq.synth_bf16((S, H), 862, 0.0, 1.0).float() * 1.25
    ids, best = mq.next_token_after_prefill(hidden, lm, fn)
    all_ids, all_best = mq.lm_head_argmax(hidden, lm, fn)  # the reference's order: every row, then slice
    torch.cuda.synchronize()
    assert ids.shape == (1,)
    assert int(ids[0]) == int(all_ids[-1]) and float(best[0]) == float(all_best[-1])
    assert mq.device_error() == 0


def test_greedy_token_in_cuda_graph():
    """One token of the loop (embedding from the fed-back ids, the step, the ids copied back)
    captured once and replayed equals the eager loop token for token."""
    H, I, V, m, T = 512, 1024, 2048, 2, 5
    layers = []
    for l in range(2):
        layers.append(mq.Layer(mq.synth_bf16((H,), 873 + 4 * l, 0.1, 0.02),
                               mq.quantize_weight(mq.synth_bf16((I, H), 870 + 4 * l, 0.0, 0.02)),
                               mq.quantize_weight(mq.synth_bf16((I, H), 871 + 4 * l, 0.0, 0.02)),
                               mq.quantize_weight(mq.synth_bf16((H, I), 872 + 4 * l, 0.0, 0.02))))
    lm = mq.quantize_weight(mq.synth_bf16((V, H), 890, 0.0, 0.02))
    fn = mq.synth_bf16((H,), 891, 0.1, 0.02)
    ids0 = torch.tensor([11, 1999], dtype=torch.int32, device="cuda")
    want = mq.GreedyLoop(layers, fn, lm, m)(ids0, T)
    loop = mq.GreedyLoop(layers, fn, lm, m)
    cur = ids0.clone()

    def token():
        mq.embed_q4(cur, lm, out=loop.h0)
        ids, _, _ = loop.step(loop.h0)
        cur.copy_(ids)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        token()  # warm-up outside capture
    torch.cuda.current_stream().wait_stream(s)
    cur.copy_(ids0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        token()
    cur.copy_(ids0)
    got = []
    for _ in range(T):
        g.replay()
        got.append(cur.clone())
    torch.cuda.synchronize()
    assert torch.equal(torch.stack(got), want)
    assert mq.device_error() == 0
