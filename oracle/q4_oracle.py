"""CPU oracle for marlin-mlx's Q4 path — TEST INFRASTRUCTURE ONLY.

Two independent restatements of the same semantics, used as the checker for the CUDA product:

* ``C`` — ctypes binding of ``oracle/libq4oracle.so`` (``q4_oracle.c``, OpenMP), the fast oracle.
* ``np_*`` functions — a NumPy mirror written from the same specification, used to cross-check the
  C oracle bit for bit on small cases.

PARITY UNPINNED: the reference delegates the arithmetic to MLX v0.25.2 (reference
``CMakeLists.txt:15-19``), which is absent here, and ships no tests or golden vectors.  Semantics
follow MLX's published affine quantization and the reference call sites cited in ``q4_oracle.h``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libq4oracle.so"

BF16, F32 = 0, 1
ROUND_HALF_EVEN, TRUE_MINMAX, NO_ZERO_SNAP, BF16_PARAMS_FIRST = 1, 2, 4, 8
GROUP = 64


# ------------------------------------------------------------------------------------------------
# bf16 helpers (bit patterns as uint16)
# ------------------------------------------------------------------------------------------------
def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(f: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_round(f: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(f))


# ------------------------------------------------------------------------------------------------
# NumPy mirror
# ------------------------------------------------------------------------------------------------
_M1, _M2 = np.uint64(0xBF58476D1CE4E5B9), np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def _mix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z ^ (z >> np.uint64(30))
        z = z * _M1
        z = z ^ (z >> np.uint64(27))
        z = z * _M2
        return z ^ (z >> np.uint64(31))


def np_synth_bf16(n: int, seed: int, mean: float, sigma: float, start: int = 0) -> np.ndarray:
    """Mirror of q4o_synth_bf16 (Irwin-Hall(12) of splitmix64 lanes, bf16 RNE)."""
    i = np.arange(start, start + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        base = _mix64(np.uint64(seed) ^ np.uint64(0x5851F42D4C957F2D))
        s = np.zeros(n, dtype=np.int64)
        for r in range(3):
            h = _mix64(base + (np.uint64(3) * i + np.uint64(r)) * _GOLD)
            for sh in (0, 16, 32, 48):
                s += ((h >> np.uint64(sh)) & np.uint64(0xFFFF)).astype(np.int64)
    z = (s - 393210).astype(np.float32)
    v = z * np.float32(np.float32(sigma) * np.float32(1.0 / 65536.0))
    v = (v + np.float32(mean)).astype(np.float32)
    return f32_to_bf16(v)


def _round(v: np.ndarray, flags: int) -> np.ndarray:
    if flags & ROUND_HALF_EVEN:
        return np.rint(v)
    a = np.abs(v).astype(np.float32)
    fl = np.floor(a)
    r = np.where(a - fl >= np.float32(0.5), fl + np.float32(1.0), fl)  # a - fl is exact
    return (np.sign(v) * r).astype(np.float32)


def np_quantize(w_bf16: np.ndarray, flags: int = 0):
    """Mirror of q4o_quantize: bf16 [N,K] -> (u32 [N,K/8], bf16 scales [N,K/64], bf16 biases)."""
    w = bf16_to_f32(w_bf16)
    N, K = w.shape
    assert K % GROUP == 0
    g = w.reshape(N, K // GROUP, GROUP)
    wmin = g.min(axis=-1)
    wmax = g.max(axis=-1)
    if not flags & TRUE_MINMAX:
        wmax = np.maximum(wmax, np.float32(0.0))
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.maximum((wmax - wmin) / np.float32(15.0), np.float32(1e-7)).astype(np.float32)
        if flags & NO_ZERO_SNAP:
            bias = wmin.astype(np.float32)
        else:
            side = np.abs(wmin) > np.abs(wmax)
            scale = np.where(side, scale, -scale).astype(np.float32)
            edge = np.where(side, wmin, wmax).astype(np.float32)
            q0 = _round((edge / scale).astype(np.float32), flags)
            nz = q0 != 0
            scale = np.where(nz, (edge / np.where(nz, q0, 1)).astype(np.float32), scale)
            bias = np.where(nz, edge, np.float32(0.0)).astype(np.float32)
    s16, b16 = f32_to_bf16(scale), f32_to_bf16(bias)
    if flags & BF16_PARAMS_FIRST:
        scale, bias = bf16_to_f32(s16), bf16_to_f32(b16)
    c = _round(((g - bias[..., None]) / scale[..., None]).astype(np.float32), flags)
    c = np.clip(c, 0, 15).astype(np.uint32).reshape(N, K // 8, 8)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    wq = np.bitwise_or.reduce(c << shifts, axis=-1).astype(np.uint32)
    return wq, s16, b16


def np_unpack(wq: np.ndarray) -> np.ndarray:
    """u32 [N, K/8] -> uint8 codes [N, K]."""
    N, W = wq.shape
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    return ((wq[..., None] >> shifts) & 15).astype(np.uint8).reshape(N, W * 8)


def np_dequant(wq, scales, biases) -> np.ndarray:
    q = np_unpack(wq).astype(np.float32)
    N, K = q.shape
    s = np.repeat(bf16_to_f32(scales), GROUP, axis=1)
    b = np.repeat(bf16_to_f32(biases), GROUP, axis=1)
    return (s * q + b).astype(np.float32)


def np_qmatmul_f64(x: np.ndarray, wq, scales, biases) -> np.ndarray:
    """Float64 reference of y = x . dequant(W)^T (tolerance checks, not bit-exact)."""
    return x.astype(np.float64) @ np_dequant(wq, scales, biases).astype(np.float64).T


# ------------------------------------------------------------------------------------------------
# ctypes binding of the C oracle
# ------------------------------------------------------------------------------------------------
class _Q4(ctypes.Structure):
    _fields_ = [("weight", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("biases", ctypes.c_void_p), ("N", ctypes.c_int64), ("K", ctypes.c_int64)]


class _Layer(ctypes.Structure):
    _fields_ = [("norm", ctypes.c_void_p), ("gate", _Q4), ("up", _Q4), ("down", _Q4)]


def build() -> Path:
    """Compile the C oracle (make -C oracle).  Returns the library path."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True,
                   env={**os.environ, "ORACLE_CC": os.environ.get("ORACLE_CC", "gcc")})
    return LIB_PATH


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class Q4:
    """A quantized tensor held in host memory (numpy arrays), MLX layout."""

    def __init__(self, weight: np.ndarray, scales: np.ndarray, biases: np.ndarray):
        self.weight = np.ascontiguousarray(weight, dtype=np.uint32)
        self.scales = np.ascontiguousarray(scales, dtype=np.uint16)
        self.biases = np.ascontiguousarray(biases, dtype=np.uint16)
        self.N, self.K = self.weight.shape[0], self.weight.shape[1] * 8

    def c(self) -> _Q4:
        return _Q4(_ptr(self.weight), _ptr(self.scales), _ptr(self.biases), self.N, self.K)


class COracle:
    def __init__(self, path: Path | None = None):
        path = Path(path or LIB_PATH)
        if not path.exists():
            build()
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        vp, i64, f32, u64, ci = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64,
                                 ctypes.c_int)
        L.q4o_synth_bf16.argtypes = [vp, i64, u64, f32, f32]
        L.q4o_synth_bf16_at.argtypes = [u64, u64, f32, f32]
        L.q4o_synth_bf16_at.restype = ctypes.c_uint16
        L.q4o_quantize.argtypes = [vp, i64, i64, ci, ci, vp, vp, vp, ctypes.c_uint]
        L.q4o_qmatmul.argtypes = [vp, ci, i64, ctypes.POINTER(_Q4), vp]
        L.q4o_rms_norm.argtypes = [vp, ci, vp, i64, i64, f32, vp]
        L.q4o_swiglu_f32.argtypes = [vp, vp, vp, i64]
        L.q4o_swiglu_bf16.argtypes = [vp, vp, vp, i64]
        L.q4o_mlp.argtypes = [vp, ci, i64, ctypes.POINTER(_Layer), vp]
        L.q4o_argmax_f32.argtypes = [vp, i64, i64, vp, vp]
        L.q4o_lm_head_argmax.argtypes = [vp, ci, i64, ctypes.POINTER(_Q4), vp, vp]
        L.q4o_decode_step.argtypes = [vp, i64, i64, ci, ctypes.POINTER(_Layer), vp,
                                      ctypes.POINTER(_Q4), f32, vp, vp, vp]
        L.q4o_num_threads.restype = ci

    # generator ----------------------------------------------------------------------------------
    def synth_bf16(self, shape, seed: int, mean: float = 0.0, sigma: float = 1.0) -> np.ndarray:
        out = np.empty(shape, dtype=np.uint16)
        self.lib.q4o_synth_bf16(_ptr(out), out.size, seed, mean, sigma)
        return out

    # operators ------------------------------------------------------------------------------------
    def quantize(self, w: np.ndarray, flags: int = 0, group_size: int = 64, bits: int = 4) -> Q4:
        w = np.ascontiguousarray(w, dtype=np.uint16)
        N, K = w.shape
        wq = np.empty((N, max(K // 8, 0)), dtype=np.uint32)
        s = np.empty((N, max(K // 64, 0)), dtype=np.uint16)
        b = np.empty_like(s)
        rc = self.lib.q4o_quantize(_ptr(w), N, K, group_size, bits, _ptr(wq), _ptr(s), _ptr(b), flags)
        if rc:
            raise ValueError(f"q4o_quantize rejected shape {w.shape} gs={group_size} bits={bits}")
        return Q4(wq, s, b)

    @staticmethod
    def _x(x: np.ndarray):
        if x.dtype == np.uint16:
            return np.ascontiguousarray(x), BF16
        return np.ascontiguousarray(x, dtype=np.float32), F32

    def qmatmul(self, x: np.ndarray, w: Q4) -> np.ndarray:
        """binary32 result; round with f32_to_bf16 for the bf16-x operator output."""
        x, dt = self._x(x)
        M = x.shape[0]
        y = np.empty((M, w.N), dtype=np.float32)
        if self.lib.q4o_qmatmul(_ptr(x), dt, M, ctypes.byref(w.c()), _ptr(y)):
            raise ValueError("q4o_qmatmul rejected its arguments")
        return y

    def rms_norm(self, x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
        x, dt = self._x(x)
        M, H = x.shape
        out = np.empty((M, H), dtype=np.float32)
        self.lib.q4o_rms_norm(_ptr(x), dt, _ptr(np.ascontiguousarray(w, np.uint16)), M, H, eps, _ptr(out))
        return out

    def swiglu_f32(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        out = np.empty_like(g)
        self.lib.q4o_swiglu_f32(_ptr(g), _ptr(u), _ptr(out), g.size)
        return out

    def swiglu_bf16(self, g, u):
        g = np.ascontiguousarray(g, np.uint16)
        u = np.ascontiguousarray(u, np.uint16)
        out = np.empty_like(g)
        self.lib.q4o_swiglu_bf16(_ptr(g), _ptr(u), _ptr(out), g.size)
        return out

    @staticmethod
    def _layer(norm, gate: Q4, up: Q4, down: Q4) -> _Layer:
        return _Layer(_ptr(norm) if norm is not None else 0, gate.c(), up.c(), down.c())

    def mlp(self, x: np.ndarray, gate: Q4, up: Q4, down: Q4) -> np.ndarray:
        x, dt = self._x(x)
        M = x.shape[0]
        y = np.empty((M, down.N), dtype=np.uint16 if dt == BF16 else np.float32)
        L = self._layer(None, gate, up, down)
        if self.lib.q4o_mlp(_ptr(x), dt, M, ctypes.byref(L), _ptr(y)):
            raise ValueError("q4o_mlp rejected its arguments")
        return y

    def lm_head_argmax(self, h: np.ndarray, lm: Q4):
        h, dt = self._x(h)
        M = h.shape[0]
        ids = np.empty(M, dtype=np.int32)
        best = np.empty(M, dtype=np.float32)
        if self.lib.q4o_lm_head_argmax(_ptr(h), dt, M, ctypes.byref(lm.c()), _ptr(ids), _ptr(best)):
            raise ValueError("q4o_lm_head_argmax rejected its arguments")
        return ids, best

    def decode_step(self, h0_bf16: np.ndarray, layers, final_norm: np.ndarray, lm: Q4,
                    eps: float = 1e-6):
        """layers: list of (norm_bf16[H], gate Q4, up Q4, down Q4).  Returns (ids, best, h32)."""
        h0 = np.ascontiguousarray(h0_bf16, dtype=np.uint16)
        M, H = h0.shape
        arr = (_Layer * len(layers))()
        keep = []
        for i, (norm, g, u, d) in enumerate(layers):
            norm = np.ascontiguousarray(norm, dtype=np.uint16)
            keep.append(norm)
            arr[i] = self._layer(norm, g, u, d)
        fn = np.ascontiguousarray(final_norm, dtype=np.uint16)
        h_out = np.empty((M, H), dtype=np.float32)
        ids = np.empty(M, dtype=np.int32)
        best = np.empty(M, dtype=np.float32)
        rc = self.lib.q4o_decode_step(_ptr(h0), M, H, len(layers), arr, _ptr(fn), ctypes.byref(lm.c()),
                                      eps, _ptr(h_out), _ptr(ids), _ptr(best))
        if rc:
            raise ValueError("q4o_decode_step rejected its arguments")
        return ids, best, h_out

    def num_threads(self) -> int:
        return self.lib.q4o_num_threads()
