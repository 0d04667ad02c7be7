"""Time the reference's own CPU path beside the numpy port — TEST INFRASTRUCTURE ONLY.

    python -m oracle.time_reference --reference-root <checkout of the reference> [--T 1 32]

Imports ``glm52_h200/reference.py`` from the given checkout, unmodified, and times one
MoE block per step through its own functions, composed as the reference's layer bench
composes its fp32 check (glm52/bench/bench_layer.py:355-374): ``add_rmsnorm`` ->
``router`` (fp32 sigmoid noaux_tc, bias, top-8, x2.5) -> ``moe_mlp`` (its per-expert
loop, bf16 linears) -> the shared expert -> ``routed + h1 + shared`` rounded to bf16.
The torch restatement that ``bench.py`` times as its reference arm and CPU baseline
(``oracle.reference_torch.moe_block``) and the numpy parity oracle
(``oracle.reference_np.moe_block``) run on the same inputs, the same cores and in the
same process: the torch restatement must match the reference bit for bit and run at its
speed; the numpy oracle is compared by max-abs over rms and its (lower) speed reported.

Inputs are the seeded GLM-5.2 block inputs of ``oracle.synth_np`` (the GPU arm's
generator). The expert stacks are allocated at full size ([256, 4096, 6144] and
[256, 6144, 2048] bf16) but only the routed experts' slices are filled: the reference's
``moe_mlp`` touches no other expert's weights, so untouched pages are never backed.

The reference tree is not shipped with this repository and does not exist on the GPU
hosts; this script runs where a checkout is present and prints one JSON line per T.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import time

import numpy as np

from . import reference_np as O
from . import reference_torch as RT
from . import synth_np as S

H, I, E, SEED = 6144, 2048, 256, 1


def _time(fn, steps: int, budget_s: float) -> tuple[float, int]:
    fn()  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    return statistics.fmean(times), len(times)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True,
                    help="directory holding glm52_h200/ of the reference checkout")
    ap.add_argument("--T", type=int, nargs="+", default=[1, 32])
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--budget-s", type=float, default=60.0)
    args = ap.parse_args()

    import torch

    sys.path.insert(0, os.path.abspath(args.reference_root))
    R = importlib.import_module("glm52_h200.reference")
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    from threadpoolctl import threadpool_limits

    threadpool_limits(cores)

    bf = torch.bfloat16
    gamma = S.make("gamma", (H,), SEED)
    gw = S.make("gate_w", (E, H), SEED)
    bias = S.make("bias", (E,), SEED)
    w13s = S.make("w13s", (2 * I, H), SEED)
    w2s = S.make("w2s", (H, I), SEED)
    w13_t = torch.empty(E, 2 * I, H, dtype=bf)
    w2_t = torch.empty(E, H, I, dtype=bf)
    filled: set[int] = set()
    gamma_t = torch.from_numpy(gamma).to(bf)
    gw_t = torch.from_numpy(gw)
    bias_t = torch.from_numpy(bias)
    w13s_t = torch.from_numpy(w13s).to(bf)
    w2s_t = torch.from_numpy(w2s).to(bf)

    for T in args.T:
        h = S.make("h", (T, H), SEED * 1000 + T)
        r = S.make("r", (T, H), SEED * 1000 + T)
        x2, _ = O.add_rmsnorm(h, r, gamma)
        _, _, ids = O.router(x2, gw, bias)
        used = sorted(set(ids.flatten().tolist()))
        w13 = {e: S.expert_weight("w13", e, H, I, SEED) for e in used}
        w2 = {e: S.expert_weight("w2", e, H, I, SEED) for e in used}
        for e in used:
            if e not in filled:
                w13_t[e] = torch.from_numpy(w13[e]).to(bf)
                w2_t[e] = torch.from_numpy(w2[e]).to(bf)
                filled.add(e)
        h_t = torch.from_numpy(h).to(bf)
        r_t = torch.from_numpy(r).to(bf)
        out_ref = {}

        def ref_step():
            with torch.no_grad():
                x2_t, h1_t = R.add_rmsnorm(h_t, r_t, gamma_t)
                _, tw, ti = R.router(x2_t, gw_t, bias_t)
                routed = R.moe_mlp(x2_t, w13_t, w2_t, tw, ti).float()
                shared = R.shared_expert_mlp(x2_t, w13s_t, w2s_t)
                out_ref["out"] = (routed + h1_t.float() + shared).to(bf)
                out_ref["ids"] = ti

        out_tor = {}

        def torch_step():
            w13d = {e: w13_t[e] for e in used}
            w2d = {e: w2_t[e] for e in used}
            out_tor.update(RT.moe_block(h_t, r_t, gamma_t, gw_t, bias_t, w13d, w2d, w13s_t,
                                        w2s_t, E))

        out_port = {}

        def port_step():
            out_port.update(O.moe_block(h, r, gamma, gw, bias, w13.__getitem__,
                                        w2.__getitem__, w13s, w2s, E))

        t_ref, n_ref = _time(ref_step, args.steps, args.budget_s)
        t_tor, n_tor = _time(torch_step, args.steps, args.budget_s)
        t_port, n_port = _time(port_step, args.steps, args.budget_s)
        o_ref = out_ref["out"].float().numpy()
        o_port = out_port["out"].astype(np.float32)
        rms = float(np.sqrt((o_ref.astype(np.float64) ** 2).mean()))
        print(json.dumps({
            "T": T, "cores": cores, "experts_routed": len(used),
            "reference_ms_per_step": t_ref * 1e3, "reference_steps": n_ref,
            "reference_tokens_per_s": T / t_ref,
            "port_ms_per_step": t_port * 1e3, "port_steps": n_port,
            "port_tokens_per_s": T / t_port,
            "port_over_reference_speed": t_ref / t_port,
            "torch_restatement_ms_per_step": t_tor * 1e3, "torch_restatement_steps": n_tor,
            "torch_restatement_over_reference_speed": t_ref / t_tor,
            "torch_restatement_bit_identical": bool(
                torch.equal(out_tor["out"], out_ref["out"])
                and torch.equal(out_tor["topk_ids"], out_ref["ids"])),
            "ids_equal": bool(np.array_equal(out_ref["ids"].numpy(), out_port["topk_ids"])),
            "out_maxabs_over_rms": float(np.abs(o_ref - o_port).max()) / rms,
            "torch_threads": torch.get_num_threads(),
        }), flush=True)


if __name__ == "__main__":
    main()
