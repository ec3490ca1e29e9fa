"""Shared helpers for the GPU parity tests (device <-> oracle conversions, error metrics)."""
from __future__ import annotations

import numpy as np
import torch

import marlin_q4 as mq
import q4_oracle as qo


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def u32(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().numpy().view(np.uint32)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().cpu().numpy()


def from_u16(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def host_q4(q: mq.QuantizedTensor) -> qo.Q4:
    return qo.Q4(u32(q.weight), u16(q.scales), u16(q.biases))


def make_q4(n: int, k: int, seed: int, sigma: float = 0.02) -> tuple[mq.QuantizedTensor, torch.Tensor]:
    w = mq.synth_bf16((n, k), seed, 0.0, sigma)
    return mq.quantize_weight(w), w


def act(shape, seed: int, dtype: torch.dtype, mean: float = 0.0, sigma: float = 1.0) -> torch.Tensor:
    x = mq.synth_bf16(shape, seed, mean, sigma)
    return x if dtype == torch.bfloat16 else x.float() * 1.25  # f32 inputs with low bits set


def host_act(x: torch.Tensor) -> np.ndarray:
    return u16(x) if x.dtype == torch.bfloat16 else f32(x)


def max_rel_row_err(y: np.ndarray, ref: np.ndarray) -> float:
    """max over rows of max|y - ref| / max|ref| (the path's float tolerance metric)."""
    y = np.asarray(y, np.float64).reshape(ref.shape[0], -1)
    ref = np.asarray(ref, np.float64).reshape(ref.shape[0], -1)
    den = np.maximum(np.abs(ref).max(axis=1), 1e-30)
    return float((np.abs(y - ref).max(axis=1) / den).max())


TOL = 1e-2  # the path's stated float tolerance: max relative error vs the fp32-accumulated reference
