"""Roofline of the MoE block, built the way the reference builds its ceilings.

glm52/traffic.py models every kernel as max(flops / C_PEAK, bytes / B_PEAK) and a chain
as the sum over its kernels (traffic.py:191-193), with bytes = algorithmic HBM traffic
and expert weights counted once per distinct expert touched (traffic.py:29-38). This
module applies that model to the block's kernels (norm, router, w13+SwiGLU, w2, merge;
the dispatch layout and permutation are counted with the activations they move), with
the measured B200 peaks of MEASURED_PEAKS.json in place of the reference's C500/H200
calibration.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
BF16, FP32, I32 = 2, 4, 4

# earlier measurement on this pool, used only when MEASURED_PEAKS.json is absent
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


@dataclass(frozen=True)
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    source: str


def peaks() -> Peaks:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return Peaks(float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                     float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return Peaks(FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback")


def expected_distinct_experts(T: int, topk: int = 8, E: int = 256) -> float:
    """E[#experts with >= 1 token] under uniform routing (glm52/traffic.py:29-38)."""
    return E * (1.0 - (1.0 - 1.0 / E) ** (T * topk))


@dataclass(frozen=True)
class KernelCost:
    name: str
    flops: float
    bytes: float


def block_kernels(T: int, ne: float, H: int = 6144, I: int = 2048, E: int = 256,
                  topk: int = 8, shared: bool = True) -> list[KernelCost]:
    """Algorithmic (flops, HBM bytes) of each kernel of one block invocation.

    ne = distinct routed experts that received >= 1 token."""
    R = T * topk
    act = T * H * BF16
    ns = 1 if shared else 0
    w13_e = 2 * I * H * BF16  # one expert's w13
    w2_e = H * I * BF16
    return [
        KernelCost("add_rmsnorm", 0.0, 4 * act + H * BF16),
        KernelCost("router", 2.0 * T * H * E, act + E * H * FP32 + T * E * FP32 + T * topk * 8),
        KernelCost("align", 0.0, T * topk * I32 * 3),
        KernelCost("w13_swiglu", 2.0 * (R + ns * T) * H * 2 * I,
                   (ne + ns) * w13_e + (R + ns * T) * H * BF16 + (R + ns * T) * I * BF16),
        KernelCost("w2", 2.0 * (R + ns * T) * I * H,
                   (ne + ns) * w2_e + (R + ns * T) * I * BF16 + (R + ns * T) * H * BF16),
        KernelCost("merge", 0.0, R * H * BF16 + (2 + ns) * act + R * FP32),
    ]


def chain_time_s(kernels: list[KernelCost], pk: Peaks, sustained: bool = False) -> float:
    c = (pk.bf16_tflops_sustained if sustained else pk.bf16_tflops) * 1e12
    b = pk.hbm_gbs * 1e9
    return sum(max(k.flops / c, k.bytes / b) for k in kernels)


def totals(kernels: list[KernelCost]) -> tuple[float, float]:
    return sum(k.flops for k in kernels), sum(k.bytes for k in kernels)


if __name__ == "__main__":
    pk = peaks()
    print(f"peaks ({pk.source}): {pk.hbm_gbs:.0f} GB/s, {pk.bf16_tflops:.0f} TF/s bf16")
    for T in (1, 32, 256, 2048, 8192):
        ne = expected_distinct_experts(T)
        ks = block_kernels(T, ne)
        f, b = totals(ks)
        t = chain_time_s(ks, pk)
        print(f"T={T:5d} ne={ne:6.1f} bytes={b/1e9:7.3f} GB flops={f/1e12:7.3f} TF "
              f"roofline={t*1e6:9.1f} us  ({T/t/1e3:9.1f} k tok/s)")
