"""On-disk Q4 weight cache in the safetensors layout, MLX's quantized-checkpoint convention.

The reference quantizes the bf16 MLP and lm_head weights at every load (src/model/weights.cpp:45-56,
:97-111, :180-194; about 2 s for the model) from safetensors shards it reads with
mx::load_safetensors (:16-35).  This module writes the quantized triplets once and reads them back
unchanged: for a quantized matrix `name`, the tensors `name.weight` (U32 [n, k/8], eight 4-bit codes
per word, low nibble first), `name.scales` and `name.biases` (BF16 [n, k/64]), the names MLX's
QuantizedLinear uses, plus any plain tensors (norm weights) under their own names.  The file
metadata records the quantization (group_size 64, bits 4, mode affine).

File layout (safetensors): u64 little-endian header length, a JSON header mapping each name to
{"dtype", "shape", "data_offsets": [begin, end]} relative to the data section (plus
"__metadata__": string -> string), padded with spaces to a multiple of 8 bytes, then the data.
Tensors are stored row-major in name order, each at an 8-byte aligned offset.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np
import torch

from .ops import Layer, QuantizedTensor

_DTYPES = {  # safetensors dtype name -> (torch dtype to view as, numpy dtype of the raw bytes)
    "U32": (torch.int32, np.uint32),
    "I32": (torch.int32, np.int32),
    "BF16": (torch.bfloat16, np.uint16),
    "F32": (torch.float32, np.float32),
}
_TORCH_TO_ST = {torch.bfloat16: "BF16", torch.float32: "F32", torch.int32: "I32"}
META = {"format": "mlx", "quantization": "affine", "group_size": "64", "bits": "4"}


def _raw(t: torch.Tensor) -> bytes:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return t.numpy().tobytes()


def save(path: str | Path, quantized: dict[str, QuantizedTensor], plain: dict[str, torch.Tensor] | None = None,
         metadata: dict[str, str] | None = None) -> None:
    """Write `quantized` (name -> QuantizedTensor) and `plain` (name -> bf16/f32/i32 tensor)."""
    entries: list[tuple[str, str, list[int], bytes]] = []
    for name, q in quantized.items():
        if q.group_size != 64 or q.bits != 4:
            raise ValueError(f"{name}: only group_size 64, bits 4 are stored")
        entries.append((f"{name}.weight", "U32", [q.n, q.k // 8], _raw(q.weight)))
        entries.append((f"{name}.scales", "BF16", [q.n, q.k // 64], _raw(q.scales)))
        entries.append((f"{name}.biases", "BF16", [q.n, q.k // 64], _raw(q.biases)))
    for name, t in (plain or {}).items():
        if t.dtype not in _TORCH_TO_ST:
            raise TypeError(f"{name}: unsupported dtype {t.dtype}")
        entries.append((name, _TORCH_TO_ST[t.dtype], list(t.shape), _raw(t)))
    entries.sort(key=lambda e: e[0])
    header: dict = {"__metadata__": dict(META, **(metadata or {}))}
    off = 0
    for name, dt, shape, data in entries:
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(data)]}
        off += len(data) + (-len(data)) % 8
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((-len(hj)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for _, _, _, data in entries:
            f.write(data)
            f.write(b"\0" * ((-len(data)) % 8))


def read_header(path: str | Path) -> tuple[dict, int]:
    """(header dict, byte offset of the data section)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if n > 100 * 2**20:
            raise ValueError("safetensors header too large")
        return json.loads(f.read(n)), 8 + n


def load(path: str | Path, device="cuda") -> tuple[dict[str, QuantizedTensor], dict[str, torch.Tensor], dict]:
    """Read a file written by `save` (or any safetensors file in MLX's quantized layout).

    Returns (quantized name -> QuantizedTensor, other tensors, metadata).  A name whose .weight is
    U32 and that has .scales and .biases becomes a QuantizedTensor; everything else is plain."""
    header, base = read_header(path)
    meta = header.pop("__metadata__", {})
    gs, bits = int(meta.get("group_size", 64)), int(meta.get("bits", 4))
    if gs != 64 or bits != 4:
        raise ValueError(f"unsupported quantization group_size={gs} bits={bits}")
    mm = np.memmap(path, dtype=np.uint8, mode="r")

    def tensor(name: str) -> torch.Tensor:
        h = header[name]
        tdt, ndt = _DTYPES[h["dtype"]]
        b0, b1 = h["data_offsets"]
        a = np.frombuffer(mm[base + b0:base + b1], dtype=ndt).reshape(h["shape"]).copy()
        return torch.from_numpy(a.view(np.int16) if ndt == np.uint16 else a.view(np.int32) if ndt == np.uint32
                                else a).view(tdt).to(device)

    quantized, plain, used = {}, {}, set()
    for name, h in header.items():
        if name.endswith(".weight") and h["dtype"] == "U32":
            stem = name[: -len(".weight")]
            if f"{stem}.scales" in header and f"{stem}.biases" in header:
                quantized[stem] = QuantizedTensor(tensor(name), tensor(f"{stem}.scales"), tensor(f"{stem}.biases"),
                                                  gs, bits)
                used.update((name, f"{stem}.scales", f"{stem}.biases"))
    for name in header:
        if name not in used:
            plain[name] = tensor(name)
    return quantized, plain, meta


def layer_prefix(i: int) -> str:
    """The reference's per-layer MLP prefix (src/model/weights.cpp:98)."""
    return f"model.language_model.layers.{i}."


def save_model(path: str | Path, layers: list[Layer], final_norm: torch.Tensor, lm: QuantizedTensor) -> None:
    """The Q4 path's weights under the reference's checkpoint names: per layer
    `...layers.{i}.mlp.{gate,up,down}_proj` and `...layers.{i}.post_attention_layernorm.weight`,
    `model.language_model.norm.weight` and the tied head as `lm_head`."""
    q, p = {"lm_head": lm}, {"model.language_model.norm.weight": final_norm}
    for i, L in enumerate(layers):
        pre = layer_prefix(i)
        q[pre + "mlp.gate_proj"], q[pre + "mlp.up_proj"], q[pre + "mlp.down_proj"] = L.gate_proj, L.up_proj, L.down_proj
        p[pre + "post_attention_layernorm.weight"] = L.post_attn_norm
    save(path, q, p)


def load_model(path: str | Path, device="cuda") -> tuple[list[Layer], torch.Tensor, QuantizedTensor]:
    """Inverse of save_model: (layers, final_norm, lm)."""
    q, p, _ = load(path, device)
    layers, i = [], 0
    while layer_prefix(i) + "mlp.gate_proj" in q:
        pre = layer_prefix(i)
        layers.append(Layer(p[pre + "post_attention_layernorm.weight"], q[pre + "mlp.gate_proj"],
                            q[pre + "mlp.up_proj"], q[pre + "mlp.down_proj"]))
        i += 1
    return layers, p["model.language_model.norm.weight"], q["lm_head"]
