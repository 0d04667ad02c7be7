"""Timing and validation helpers with the reference's semantics (glm52/common.py).

* `bench_chain`: a chain of launches timed as ONE unit, one L2 flush before each
  repetition of the whole chain, never between its kernels (glm52/common.py:73-122);
  CUDA events on the current stream; p50/p10/p90 plus a no-flush p50.
* `rel_err` / `check`: max-abs error over max|ref| against a tolerance
  (glm52/common.py:186-203).
* `record`: JSON result with device metadata (glm52/common.py:206-220).
"""

from __future__ import annotations

import json
import os
import statistics
import time
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Callable, Sequence

import torch

RESULTS_DIR = Path(os.environ.get("FUSION_B200_RESULTS_DIR",
                                  Path(__file__).resolve().parent.parent / "results"))
_flush_buf: torch.Tensor | None = None


def flush_l2() -> None:
    global _flush_buf
    if _flush_buf is None:
        l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
        _flush_buf = torch.empty(max(128 * 2**20, 4 * l2), dtype=torch.uint8, device="cuda")
    _flush_buf.zero_()


@dataclass
class Timing:
    p50_ms: float
    p10_ms: float
    p90_ms: float
    mean_ms: float
    n: int
    noflush_p50_ms: float = float("nan")

    def as_dict(self) -> dict:
        return asdict(self)


def bench_chain(fns: Sequence[Callable[[], object]] | Callable[[], object], warmup: int = 25,
                rep: int = 100, flush: bool = True) -> Timing:
    if callable(fns):
        fns = [fns]
    for _ in range(warmup):
        for fn in fns:
            fn()
    torch.cuda.synchronize()

    def measure(do_flush: bool) -> list[float]:
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(rep)]
        for a, b in ev:
            if do_flush:
                flush_l2()
            a.record()
            for fn in fns:
                fn()
            b.record()
        torch.cuda.synchronize()
        return sorted(a.elapsed_time(b) for a, b in ev)

    t = measure(flush)
    nf = measure(False)
    n = len(t)
    return Timing(t[n // 2], t[max(0, int(0.1 * n))], t[min(n - 1, int(0.9 * n))],
                  statistics.fmean(t), n, nf[len(nf) // 2])


def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    g, r = got.float(), ref.float()
    return ((g - r).abs().max() / r.abs().max().clamp_min(1e-6)).item()


def check(got: torch.Tensor, ref: torch.Tensor, tol: float = 2e-2, label: str = "") -> dict:
    err = rel_err(got, ref)
    ok = err <= tol and bool(torch.isfinite(got).all().item())
    return {"label": label, "rel_err": err, "tol": tol, "ok": ok}


def record(name: str, payload: dict) -> Path:
    RESULTS_DIR.mkdir(parents=True, exist_ok=True)
    path = RESULTS_DIR / f"{name}.json"
    payload = dict(payload)
    payload.setdefault("_meta", {}).update({
        "recorded_at": time.strftime("%Y-%m-%d %H:%M:%S"),
        "device": torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu",
        "visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES", "all"),
        "torch": torch.__version__,
    })
    path.write_text(json.dumps(payload, indent=2, default=str))
    return path
