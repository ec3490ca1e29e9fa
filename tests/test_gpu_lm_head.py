"""GPU parity: fused Q4 lm_head + greedy argmax (src/model/marlin.cpp:161-169, sampler.cpp:14-16).

Token ids must be bit-exact against the oracle, including vocabulary sharding with the packed-key
max merge and the first-index tie rule."""
import numpy as np
import pytest
import torch

import marlin_q4 as mq
import q4_oracle as qo
from gpu_util import act, from_u16, host_act, host_q4, make_q4, u16

pytestmark = pytest.mark.gpu

V, H = 248320, 2048


@pytest.fixture(scope="module")
def lm():
    q, w = make_q4(V, H, 3)
    norm = mq.synth_bf16((H,), 4, 0.1, 0.02)
    return q, host_q4(q), norm, u16(norm)


@pytest.mark.parametrize("m", [1, 2, 5, 8, 10, 13])
def test_lm_head_argmax_after_final_norm(oracle, lm, m):
    """Config 3: hidden bf16 ~N(0,1) -> RMSNorm(1+w) (binary32, as the reference's C++ evaluates it)
    -> Q4 lm_head -> argmax."""
    q, hq, norm, hn = lm
    h = act((m, H), 10 + m, torch.bfloat16)
    ids, best = mq.lm_head_argmax(h, q, norm_weight=norm)
    p = oracle.rms_norm(host_act(h), hn)
    rids, rbest = oracle.lm_head_argmax(p, hq)
    assert np.array_equal(ids.cpu().numpy(), rids)
    assert np.allclose(best.cpu().numpy(), rbest, rtol=1e-5)
    assert mq.device_error() == 0


@pytest.mark.parametrize("dtype,m", [(torch.bfloat16, 4), (torch.float32, 4), (torch.bfloat16, 32),
                                     (torch.float32, 10), (torch.bfloat16, 33)])
def test_lm_head_argmax_plain(oracle, lm, dtype, m):
    """No norm: bf16 hidden compares bf16-rounded logits (ties -> first index); f32 compares f32."""
    q, hq = lm[0], lm[1]
    h = act((m, H), 30 + m, dtype)
    ids, best = mq.lm_head_argmax(h, q)
    rids, rbest = oracle.lm_head_argmax(host_act(h), hq)
    assert np.array_equal(ids.cpu().numpy(), rids)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_vocab_sharded_argmax(oracle, lm, tp):
    q, hq, norm, hn = lm
    h = act((3, H), 40 + tp, torch.bfloat16)
    full_ids, _ = mq.lm_head_argmax(h, q, norm_weight=norm)
    shard = V // tp
    keys = [mq.lm_head_argmax(h, q.shard_rows(r * shard, (r + 1) * shard), norm_weight=norm,
                              vocab_offset=r * shard, want_keys=True) for r in range(tp)]
    # keys are unsigned: compare as uint64
    merged = np.stack([k.cpu().numpy().view(np.uint64) for k in keys]).max(axis=0)
    ids, _ = mq.decode_keys(torch.from_numpy(merged.view(np.int64)).cuda())
    assert torch.equal(ids, full_ids)


def test_ties_take_first_index():
    """Identical weight rows give identical logits; the lowest index wins."""
    k = 256
    n = 40000
    h = act((1, k), 5, torch.float32)
    base = torch.zeros((n, k), dtype=torch.float32, device="cuda")
    base += 0.001 * act((n, k), 6, torch.float32)
    hot = (h[0] / h[0].norm()) * 0.5
    for r in (30001, 777, 5003):
        base[r] = hot
    q = mq.quantize_weight(base.to(torch.bfloat16))
    ids, best = mq.lm_head_argmax(h, q)
    assert ids.item() == 777
    # all three rows are bit-identical after quantization
    assert torch.equal(q.weight[777], q.weight[30001]) and torch.equal(q.weight[777], q.weight[5003])


def test_ragged_vocab_and_workspace_reuse(oracle):
    q, _ = make_q4(1003, 512, 8)
    hq = host_q4(q)
    ws = mq.LmHeadWorkspace(3, "cuda")
    for seed in range(3):
        h = act((3, 512), 60 + seed, torch.float32)
        ids, _ = mq.lm_head_argmax(h, q, workspace=ws)
        rids, _ = oracle.lm_head_argmax(host_act(h), hq)
        assert np.array_equal(ids.cpu().numpy(), rids)
        assert int(ws.buf.count_nonzero()) == 0  # the call leaves its workspace zeroed


def test_all_equal_logits_pick_index_zero():
    q = mq.quantize_weight(torch.zeros((999, 128), dtype=torch.bfloat16, device="cuda"))
    ids, best = mq.lm_head_argmax(act((2, 128), 1, torch.float32), q)
    assert ids.tolist() == [0, 0]
