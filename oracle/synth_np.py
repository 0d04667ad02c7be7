"""Seeded synthetic inputs in pure numpy — TEST INFRASTRUCTURE ONLY.

A host restatement of the library's generator (``fusion_b200/csrc/synth.cu``:
splitmix64 finaliser -> twelve 16-bit uniforms -> Irwin-Hall(12) normal, one IEEE fp32
rounding per multiply and add, bf16 by round-to-nearest-even). It exists so that the CPU
arms of ``bench.py`` (the reference timing and the CPU baseline) build their inputs
without loading the CUDA library: the reference arm must run nothing of the product.
``tests/test_oracle_golden.py`` pins it bit-for-bit against ``fus_synth_fill_host``.

Stream names, seeds and distributions are the ones ``fusion_b200/synth.py`` uses.
"""

from __future__ import annotations

import concurrent.futures as cf
import os

import numpy as np

from .reference_np import bf16

# name -> (stream id, mean, std, is_bf16)   (same table as fusion_b200/synth.py STREAMS)
STREAMS = {
    "h": (1, 0.0, 1.0, True),
    "r": (2, 0.0, 1.0, True),
    "gamma": (3, 1.0, 0.02, True),
    "gate_w": (4, 0.0, 0.02, False),
    "bias": (5, 0.0, 1e-3, False),
    "w13": (6, 0.0, 0.02, True),
    "w2": (7, 0.0, 0.02, True),
    "w13s": (8, 0.0, 0.02, True),
    "w2s": (9, 0.0, 0.02, True),
}

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _stream_key(seed: int) -> np.uint64:
    with np.errstate(over="ignore"):
        return _mix64(np.array([seed], dtype=np.uint64) + _GOLDEN)[0]


def stream_seed(base_seed: int, name: str) -> int:
    return base_seed * 1_000_003 + STREAMS[name][0]


def _fill_chunk(key: np.uint64, offset: int, n: int, mean: float, std: float,
                as_bf16: bool) -> np.ndarray:
    i = np.arange(offset, offset + n, dtype=np.uint64)
    s = np.zeros(n, dtype=np.int64)
    m16 = np.uint64(0xFFFF)
    with np.errstate(over="ignore"):
        for j in range(3):
            h = _mix64(key + (np.uint64(3) * i + np.uint64(j)) * _GOLDEN)
            s += (h & m16).astype(np.int64)
            s += ((h >> np.uint64(16)) & m16).astype(np.int64)
            s += ((h >> np.uint64(32)) & m16).astype(np.int64)
            s += (h >> np.uint64(48)).astype(np.int64)
    z = (s - 393210).astype(np.float32) * np.float32(1.0 / 65536.0)
    v = z * np.float32(std)
    v = v + np.float32(mean)
    return bf16(v) if as_bf16 else v


def make(name: str, shape, base_seed: int, offset: int = 0, threads: int | None = None,
         chunk: int = 1 << 20) -> np.ndarray:
    """Stream `name` of config `base_seed`, elements [offset, offset + prod(shape)), as a
    float32 array (bf16-valued for the bf16 streams)."""
    _, mean, std, as_bf16 = STREAMS[name]
    key = _stream_key(stream_seed(base_seed, name))
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    starts = list(range(0, n, chunk))

    def work(b: int) -> None:
        e = min(n, b + chunk)
        out[b:e] = _fill_chunk(key, offset + b, e - b, mean, std, as_bf16)

    nt = threads or min(32, os.cpu_count() or 1)
    if nt > 1 and len(starts) > 1:
        with cf.ThreadPoolExecutor(nt) as ex:
            list(ex.map(work, starts))
    else:
        for b in starts:
            work(b)
    return out.reshape(shape)


def expert_weight(name: str, e: int, H: int, I: int, base_seed: int) -> np.ndarray:
    """Routed expert e's w13 [2I, H] or w2 [H, I] from its offset in the [E, ...] stack."""
    shape = (2 * I, H) if name == "w13" else (H, I)
    return make(name, shape, base_seed, offset=e * shape[0] * shape[1])
