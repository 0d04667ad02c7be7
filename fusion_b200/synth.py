"""Seeded synthetic inputs for the GLM-5.2 MoE block.

Every tensor is one stream of the library's bit-reproducible generator
(``fus_synth_fill`` on the GPU, ``fus_synth_fill_host`` on the CPU give the same
bits), so the CPU oracle and the GPU see identical inputs without copying 19 GB of
expert weights, and the oracle can regenerate just the experts a batch routes to.

Distributions follow the configs: h, r ~ N(0,1) bf16; gamma = 1 + N(0, 0.02) bf16;
router W_g ~ N(0, 0.02) fp32; e_score_correction_bias ~ N(0, 1e-3) fp32; expert and
shared weights ~ N(0, 0.02) bf16. "N" is the generator's Irwin-Hall(12) normal.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops

# name -> (stream id, mean, std, dtype)
STREAMS: dict[str, tuple[int, float, float, torch.dtype]] = {
    "h": (1, 0.0, 1.0, torch.bfloat16),
    "r": (2, 0.0, 1.0, torch.bfloat16),
    "gamma": (3, 1.0, 0.02, torch.bfloat16),
    "gate_w": (4, 0.0, 0.02, torch.float32),
    "bias": (5, 0.0, 1e-3, torch.float32),
    "w13": (6, 0.0, 0.02, torch.bfloat16),
    "w2": (7, 0.0, 0.02, torch.bfloat16),
    "w13s": (8, 0.0, 0.02, torch.bfloat16),
    "w2s": (9, 0.0, 0.02, torch.bfloat16),
    "a_attn": (10, 0.0, 0.05, torch.bfloat16),  # attention output entering o_proj
    "w_o": (11, 0.0, 0.02, torch.bfloat16),     # o_proj weight [K, H]
}


def stream_seed(base_seed: int, name: str) -> int:
    return base_seed * 1_000_003 + STREAMS[name][0]


def fill(t: torch.Tensor, base_seed: int, name: str, offset: int = 0) -> torch.Tensor:
    _, mean, std, dtype = STREAMS[name]
    assert t.dtype == dtype, (name, t.dtype, dtype)
    return ops.synth_fill(t, stream_seed(base_seed, name), mean, std, offset)


def make(name: str, shape, base_seed: int, device="cpu", offset: int = 0) -> torch.Tensor:
    t = torch.empty(*shape, dtype=STREAMS[name][3], device=device)
    return fill(t, base_seed, name, offset)


@dataclass(frozen=True)
class Dims:
    H: int = 6144
    I: int = 2048
    E: int = 256
    topk: int = 8


def expert_weight(name: str, e: int, dims: Dims, base_seed: int, device="cpu") -> torch.Tensor:
    """One routed expert's w13 [2I, H] or w2 [H, I], regenerated from its offset in the
    full [E, ...] stack."""
    shape = (2 * dims.I, dims.H) if name == "w13" else (dims.H, dims.I)
    n = shape[0] * shape[1]
    return make(name, shape, base_seed, device, offset=e * n)


def make_block_weights(base_seed: int, dims: Dims = Dims(), device="cuda",
                       shared: bool = True) -> dict[str, torch.Tensor]:
    """All block weights of config ``base_seed`` (19.3 GB of expert weights at GLM dims;
    generated on the device in a few milliseconds)."""
    d = dims
    w = {
        "gamma": make("gamma", (d.H,), base_seed, device),
        "gate_w": make("gate_w", (d.E, d.H), base_seed, device),
        "bias": make("bias", (d.E,), base_seed, device),
        "w13": make("w13", (d.E, 2 * d.I, d.H), base_seed, device),
        "w2": make("w2", (d.E, d.H, d.I), base_seed, device),
    }
    if shared:
        w["w13s"] = make("w13s", (2 * d.I, d.H), base_seed, device)
        w["w2s"] = make("w2s", (d.H, d.I), base_seed, device)
    return w


def make_inputs(base_seed: int, T: int, dims: Dims = Dims(), device="cuda"):
    return make("h", (T, dims.H), base_seed, device), make("r", (T, dims.H), base_seed, device)


def zipf_bias_np(E: int, s: float, c: float, perm_seed: int):
    """e_score_correction_bias giving Zipf(s) expert popularity:
    b[pi(i)] = c * log(p_i), p_i = i^-s / sum, pi a seeded permutation (numpy, fp32)."""
    import numpy as np

    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    p /= p.sum()
    perm = np.random.default_rng(perm_seed).permutation(E)
    b = np.empty(E, dtype=np.float64)
    b[perm] = c * np.log(p)
    return b.astype(np.float32)


def zipf_bias(device="cpu") -> torch.Tensor:
    """The calibrated config-4 bias (scale c fitted by tests/golden/calibrate_zipf.py)."""
    import json
    from pathlib import Path

    cfg = json.loads((Path(__file__).resolve().parent / "zipf_bias.json").read_text())
    b = zipf_bias_np(256, cfg["s"], cfg["c"], cfg["perm_seed"])
    return torch.from_numpy(b).to(device)
