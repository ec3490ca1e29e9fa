"""CPU tests of the C ABI boundary: the product library loads, exports exactly what
include/marlin_q4.h declares, and rejects bad arguments before touching the GPU."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "marlin_q4.h"


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(marlin_q4_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from marlin_q4 import _lib
    return _lib.load()


def test_header_and_binding_agree():
    from marlin_q4 import _lib
    assert declared_functions() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_exported_symbols_are_c_linkage():
    import subprocess
    from marlin_q4 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    for name in declared_functions():
        assert name in exported, name


def test_version_and_status_strings(lib):
    assert b"sm_100a" in lib.marlin_q4_version()
    assert lib.marlin_q4_status_string(0) == b"ok"
    assert b"shape" in lib.marlin_q4_status_string(-2)


def test_workspace_sizes(lib):
    assert lib.marlin_q4_lm_head_workspace_size(1) >= 16
    assert lib.marlin_q4_lm_head_workspace_size(0) == 0
    assert lib.marlin_q4_mlp_workspace_size(4, 6144, 1) >= 4 * 6144 * 4
    assert lib.marlin_q4_decode_step_workspace_size(1, 2048, 6144) >= 4 * (2048 + 6144)


def _tensor(n, k, gs=64, bits=4, ptr=0x10000):
    from marlin_q4._lib import Q4Tensor
    return Q4Tensor(ptr, ptr + 0x100000, ptr + 0x200000, n, k, gs, bits)


def test_argument_validation_without_gpu(lib):
    """Invalid arguments are rejected before any CUDA call (no device needed)."""
    from marlin_q4 import _lib as L
    fake = 0x10000  # never dereferenced: every call below fails validation first
    assert lib.marlin_q4_quantize(None, 8, 64, 64, 4, fake, fake, fake, None) == L.ERR_ARG
    assert lib.marlin_q4_decode_step_kernels(0, 2048, 6144, 24) == L.ERR_ARG
    assert lib.marlin_q4_decode_step_kernels(1, 2048, 6144, 0) == L.ERR_ARG
    assert lib.marlin_q4_set_step_kernels(7) == L.ERR_ARG
    assert lib.marlin_q4_quantize(fake, 8, 96, 64, 4, fake, fake, fake, None) == L.ERR_SHAPE
    assert lib.marlin_q4_quantize(fake, 8, 64, 32, 4, fake, fake, fake, None) == L.ERR_SHAPE
    assert lib.marlin_q4_quantize(fake, 8, 64, 64, 8, fake, fake, fake, None) == L.ERR_SHAPE
    assert lib.marlin_q4_quantize(fake + 2, 8, 64, 64, 4, fake, fake, fake, None) == L.ERR_ALIGN
    t = _tensor(16, 64)
    assert lib.marlin_q4_matmul(fake, 0, 0, ctypes.byref(t), fake, None) == L.ERR_ARG
    assert lib.marlin_q4_matmul(fake, 7, 1, ctypes.byref(t), fake, None) == L.ERR_ARG
    assert lib.marlin_q4_matmul(fake + 1, 0, 1, ctypes.byref(t), fake, None) == L.ERR_ALIGN
    bad = _tensor(16, 96)
    assert lib.marlin_q4_matmul(fake, 0, 1, ctypes.byref(bad), fake, None) == L.ERR_SHAPE
    bad = _tensor(16, 64, gs=128)
    assert lib.marlin_q4_matmul(fake, 0, 1, ctypes.byref(bad), fake, None) == L.ERR_SHAPE
    mis = _tensor(16, 64, ptr=0x10004)
    assert lib.marlin_q4_matmul(fake, 0, 1, ctypes.byref(mis), fake, None) == L.ERR_ALIGN
    g, u, d = _tensor(128, 64), _tensor(128, 64), _tensor(64, 128)
    bad_d = _tensor(64, 192)
    assert lib.marlin_q4_mlp(fake, 0, 1, ctypes.byref(g), ctypes.byref(u), ctypes.byref(bad_d), fake, fake,
                             1 << 20, None) == L.ERR_SHAPE
    assert lib.marlin_q4_mlp(fake, 0, 1, ctypes.byref(g), ctypes.byref(u), ctypes.byref(d), fake, fake,
                             4, None) == L.ERR_WORKSPACE
    lm = _tensor(1000, 64)
    assert lib.marlin_q4_lm_head_argmax(fake, 0, 1, None, 1e-6, ctypes.byref(lm), 0, None, None, None, fake,
                                        64, None) == L.ERR_ARG
    assert lib.marlin_q4_lm_head_argmax(fake, 0, 1, None, 1e-6, ctypes.byref(lm), 0, fake, None, None, None,
                                        64, None) == L.ERR_WORKSPACE
    assert lib.marlin_q4_decode_step(fake, 1, 64, 0, None, fake, 1e-6, ctypes.byref(lm), fake, None, None, fake,
                                     1 << 20, None) == L.ERR_ARG
    assert lib.marlin_q4_synth_bf16(None, 10, 1, 0.0, 1.0, None) == L.ERR_ARG


def test_python_front_end_refuses_cpu_tensors():
    import torch
    import marlin_q4
    with pytest.raises(ValueError):
        marlin_q4.quantize_weight(torch.zeros(8, 64, dtype=torch.bfloat16))


def test_host_decode_step_refuses_unpinned_buffers():
    import types

    import torch
    import marlin_q4
    fake = types.SimpleNamespace(m=2, hidden=64, ids=torch.zeros(2, dtype=torch.int32))
    with pytest.raises(ValueError):
        marlin_q4.HostDecodeStep(fake, torch.zeros(2, 64, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.int32))
