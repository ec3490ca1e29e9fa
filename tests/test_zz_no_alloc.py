"""marlin_q4_lm_head_argmax_static: the lm_head + argmax entry point that takes no workspace.

It keeps its keys in a library-owned device array shared by all calls on a device, so these tests
call it twice in a row (the second call relies on the first leaving the array zeroed) and compare
both results with marlin_q4_lm_head_argmax, which uses a caller workspace.  Kept in its own file,
collected last, so it runs after the other GPU tests as well as alone."""
import ctypes

import numpy as np
import pytest
import torch

import marlin_q4 as mq
from marlin_q4 import _lib

MAX_ROWS = 64  # MARLIN_Q4_LM_HEAD_STATIC_MAX_ROWS
N, H = 31040, 2048  # one vocabulary shard of the 248320-row lm_head at tp = 8


def _static_call(lib, h, q, norm, vocab_offset=0):
    m = h.shape[0]
    ids = torch.empty(m, dtype=torch.int32, device=h.device)
    best = torch.empty(m, dtype=torch.float32, device=h.device)
    keys = torch.empty(m, dtype=torch.int64, device=h.device)
    tl = q.c()
    rc = lib.marlin_q4_lm_head_argmax_static(
        h.data_ptr(), 0 if h.dtype == torch.bfloat16 else 1, m, norm.data_ptr() if norm is not None else None,
        1e-6, ctypes.byref(tl), vocab_offset, ids.data_ptr(), best.data_ptr(), keys.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.marlin_q4_status_string(rc)
    return ids, best, keys


def test_static_rejects_rows_beyond_limit():
    """m above the scratch array's capacity is refused before any CUDA call (no GPU needed)."""
    lib = _lib.load()
    t = _lib.Q4Tensor(0x10000, 0x20000, 0x30000, 128, 64, 64, 4)
    fake = 0x40000  # never dereferenced
    assert lib.marlin_q4_lm_head_argmax_static(fake, 0, MAX_ROWS + 1, None, 1e-6, ctypes.byref(t), 0, fake,
                                               None, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.marlin_q4_lm_head_argmax_static(fake, 0, 0, None, 1e-6, ctypes.byref(t), 0, fake,
                                               None, None, None) == _lib.ERR_ARG


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,m,normed", [(torch.bfloat16, 3, True), (torch.bfloat16, MAX_ROWS, False),
                                            (torch.float32, 12, True)])
def test_static_matches_workspace_entry_point(dtype, m, normed):
    lib = _lib.load()
    w = mq.synth_bf16((N, H), 71, 0.0, 0.02)
    q = mq.quantize_weight(w)
    norm = mq.synth_bf16((H,), 72, 0.1, 0.02) if normed else None
    h = mq.synth_bf16((m, H), 73 + m, 0.0, 1.0)
    if dtype == torch.float32:
        h = h.float() * 1.25
    ref_ids, ref_best = mq.lm_head_argmax(h, q, norm_weight=norm, vocab_offset=5)
    for _ in range(2):  # the second call needs the first to have left the shared keys zeroed
        ids, best, keys = _static_call(lib, h, q, norm, vocab_offset=5)
        torch.cuda.synchronize()
        assert torch.equal(ids, ref_ids)
        assert np.allclose(best.cpu().numpy(), ref_best.cpu().numpy(), rtol=1e-6, atol=0.0)
        dec_ids, _ = mq.decode_keys(keys)
        assert torch.equal(dec_ids, ref_ids)
    assert mq.device_error() == 0
