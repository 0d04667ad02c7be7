"""Checkpoint ingest: one MoE layer of a Hugging Face checkpoint into the block's layout.

The block keeps sglang's FusedMoE layout (glm52/config.py:61-64; glm52_h200/reference.py
:36-39): w13 [E, 2I, H] with the gate rows first and the up rows second, w2 [E, H, I],
the shared expert as w13s [2I, H] / w2s [H, I], the router weight [E, H] (fp32, split
into bf16 planes by MoEBlock) and its e_score_correction_bias [E].

Hugging Face names of a GLM-4.5/5 (Glm4Moe) or DeepSeek-V3 MoE layer L:

    model.layers.L.post_attention_layernorm.weight             gamma [H]
    model.layers.L.mlp.gate.weight                             router [E, H]
    model.layers.L.mlp.gate.e_score_correction_bias            bias [E]
    model.layers.L.mlp.experts.e.{gate,up,down}_proj.weight    [I,H] [I,H] [H,I]
    model.layers.L.mlp.shared_experts.{gate,up,down}_proj.weight

FP8 checkpoints store a linear weight as float8_e4m3fn plus `<name>_scale_inv` (fp32,
one scale per 128 x 128 block); those are dequantised to bf16 on the device at load
(fus_fp8_block_dequant). Expert stacks are filled one expert at a time, so no
stack-sized temporary exists.

`read_safetensors(path)` reads the .safetensors container (8-byte little-endian header
length, JSON header of dtype / shape / byte offsets, raw little-endian data) without the
safetensors package.
"""

from __future__ import annotations

import json
import struct
from collections.abc import Mapping
from pathlib import Path

import numpy as np
import torch

from . import ops

_ST_DTYPES = {
    "BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32,
    "F8_E4M3": torch.float8_e4m3fn, "I32": torch.int32, "I64": torch.int64, "U8": torch.uint8,
}


def read_safetensors(path: str | Path, names=None) -> dict[str, torch.Tensor]:
    """Tensors of a .safetensors file (all, or those in `names`) as CPU tensors."""
    path = Path(path)
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, meta in header.items():
            if name == "__metadata__" or (names is not None and name not in names):
                continue
            dt = _ST_DTYPES.get(meta["dtype"])
            if dt is None:
                raise ValueError(f"{name}: safetensors dtype {meta['dtype']} not supported")
            b, e = meta["data_offsets"]
            f.seek(base + b)
            raw = bytearray(f.read(e - b))
            t = torch.frombuffer(raw, dtype=torch.uint8) if e > b else torch.empty(0, dtype=torch.uint8)
            out[name] = t.view(dt).reshape(meta["shape"]).clone()
    return out


def write_safetensors(path: str | Path, tensors: Mapping[str, torch.Tensor]) -> None:
    """The inverse of read_safetensors (used to build test checkpoints)."""
    rev = {v: k for k, v in _ST_DTYPES.items()}
    header, blobs, off = {}, [], 0
    for name, t in tensors.items():
        t = t.detach().cpu().contiguous()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": rev[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def layer_keys(layer: int, E: int, shared: bool = True) -> dict[str, str]:
    p = f"model.layers.{layer}."
    k = {"gamma": p + "post_attention_layernorm.weight", "gate_w": p + "mlp.gate.weight",
         "bias": p + "mlp.gate.e_score_correction_bias"}
    for e in range(E):
        for part in ("gate", "up", "down"):
            k[f"e{e}.{part}"] = p + f"mlp.experts.{e}.{part}_proj.weight"
    if shared:
        for part in ("gate", "up", "down"):
            k[f"s.{part}"] = p + f"mlp.shared_experts.{part}_proj.weight"
    return k


def _to_bf16(sd: Mapping[str, torch.Tensor], name: str, out: torch.Tensor) -> None:
    """Copy checkpoint tensor `name` into the bf16 device view `out` (FP8 dequantised)."""
    t = sd[name]
    if tuple(t.shape) != tuple(out.shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(out.shape)}")
    if t.dtype == torch.float8_e4m3fn:
        scale = sd.get(name + "_scale_inv")
        if scale is None:
            raise ValueError(f"{name}: FP8 weight without {name}_scale_inv")
        src = t.to(out.device, non_blocking=True)
        sc = scale.to(device=out.device, dtype=torch.float32)
        br = -(-t.shape[0] // sc.shape[0])
        bc = -(-t.shape[1] // sc.shape[1])
        ops.fp8_block_dequant(src, sc, out, (br, bc))
    else:
        out.copy_(t.to(torch.bfloat16) if t.dtype != torch.bfloat16 else t, non_blocking=True)


def load_moe_layer(sd: Mapping[str, torch.Tensor], layer: int, *, E: int, H: int, I: int,
                   device="cuda", shared: bool = True) -> dict[str, torch.Tensor]:
    """Block weights of MoE layer `layer` from a state dict (name -> tensor, e.g. the
    union of read_safetensors over the checkpoint's shards) in the block's layout, on
    `device`: gamma, gate_w (fp32), bias (fp32), w13, w2 (+ w13s, w2s)."""
    k = layer_keys(layer, E, shared)
    dev = torch.device(device)
    bf = torch.bfloat16
    out = {
        "gamma": torch.empty(H, dtype=bf, device=dev),
        "gate_w": sd[k["gate_w"]].to(device=dev, dtype=torch.float32),
        "bias": sd[k["bias"]].to(device=dev, dtype=torch.float32),
        "w13": torch.empty(E, 2 * I, H, dtype=bf, device=dev),
        "w2": torch.empty(E, H, I, dtype=bf, device=dev),
    }
    if tuple(out["gate_w"].shape) != (E, H) or tuple(out["bias"].shape) != (E,):
        raise ValueError("router weight / bias shape does not match E, H")
    _to_bf16(sd, k["gamma"], out["gamma"])
    for e in range(E):  # gate rows [0, I), up rows [I, 2I): sglang's w13
        _to_bf16(sd, k[f"e{e}.gate"], out["w13"][e, :I])
        _to_bf16(sd, k[f"e{e}.up"], out["w13"][e, I:])
        _to_bf16(sd, k[f"e{e}.down"], out["w2"][e])
    if shared:
        out["w13s"] = torch.empty(2 * I, H, dtype=bf, device=dev)
        out["w2s"] = torch.empty(H, I, dtype=bf, device=dev)
        _to_bf16(sd, k["s.gate"], out["w13s"][:I])
        _to_bf16(sd, k["s.up"], out["w13s"][I:])
        _to_bf16(sd, k["s.down"], out["w2s"])
    return out


def fp8_quantize_blocks(w: np.ndarray, block=(128, 128)) -> tuple[torch.Tensor, np.ndarray]:
    """Block-scaled e4m3 quantisation as FP8 checkpoints store it (scale = amax / 448 per
    block, value = e4m3(w / scale)): (e4m3 CPU tensor, fp32 scales), for test checkpoints."""
    R, C = w.shape
    br, bc = block
    sr, sc = -(-R // br), -(-C // bc)
    scale = np.zeros((sr, sc), dtype=np.float32)
    q = np.zeros_like(w, dtype=np.float32)
    for i in range(sr):
        for j in range(sc):
            blk = w[i * br:(i + 1) * br, j * bc:(j + 1) * bc]
            s = max(float(np.abs(blk).max()) / 448.0, 1e-12)
            scale[i, j] = s
            q[i * br:(i + 1) * br, j * bc:(j + 1) * bc] = blk / s
    q8 = torch.from_numpy(q).to(torch.float8_e4m3fn)
    return q8, scale
