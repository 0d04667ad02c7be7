"""Calibrate the Zipf(1.1) routing skew of BASELINE config 4.

The correction bias is b[pi(i)] = c * log(p_i), p_i ~ 1 / i^1.1 over a seeded permutation
pi of the 256 experts. For candidate scales c this routes T=8192 seeded tokens through
the fp32 router (CPU oracle) and fits the log-log slope of expert load vs. popularity
rank; the c whose slope is closest to -1.1 is written to fusion_b200/zipf_bias.json, which
fusion_b200.synth.zipf_bias reads back.

    python tests/golden/calibrate_zipf.py
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from fusion_b200 import synth  # noqa: E402
from oracle import reference_np as O  # noqa: E402


def slope(counts: np.ndarray) -> float:
    c = np.sort(counts)[::-1].astype(np.float64)
    k = np.arange(1, c.size + 1)
    keep = c > 0
    return float(np.polyfit(np.log(k[keep][:128]), np.log(c[keep][:128]), 1)[0])


def main() -> None:
    d = synth.Dims()
    T, s_zipf, perm_seed = 8192, 1.1, 4
    x2 = synth.make("h", (T, d.H), 4000).float().numpy()
    gw = synth.make("gate_w", (d.E, d.H), 4).numpy()
    logits = O.router_logits(x2, gw)
    best = None
    for c in np.round(np.arange(0.03, 0.151, 0.005), 3):
        bias = synth.zipf_bias_np(d.E, s_zipf, float(c), perm_seed)
        _, ids = O.router_select(logits, bias)
        sl = slope(np.bincount(ids.reshape(-1), minlength=d.E))
        print(f"c={c:.3f} slope={sl:.3f}")
        if best is None or abs(sl + s_zipf) < abs(best[1] + s_zipf):
            best = (float(c), sl)
    out = {"s": s_zipf, "c": best[0], "perm_seed": perm_seed, "fitted_slope": best[1],
           "T": T, "fit": "top-128 experts by load, log-log least squares"}
    (HERE.parent.parent / "fusion_b200" / "zipf_bias.json").write_text(json.dumps(out, indent=1) + "\n")
    print(out)


if __name__ == "__main__":
    main()
