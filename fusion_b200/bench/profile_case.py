"""Small, self-contained grouped-GEMM launches for ncu captures.

    python -m fusion_b200.bench.profile_case decode  [reps]
    python -m fusion_b200.bench.profile_case prefill [reps]
    python -m fusion_b200.bench.profile_case prefill32 [reps]
    python -m fusion_b200.bench.profile_case block8192 [reps]   (any block<T>)

decode : the w13+SwiGLU and w2 launches of the decode block at T=1 — 8 routed experts
         with one token each plus the shared expert (the same tile shapes, flags and
         bytes per launch as the block), on a 16-expert weight stack (1.2 GB allocated).
prefill: 16 experts x 256 tokens each (the per-expert load of T=8192 over 256 experts),
         256-token tiles with two weight tiles per CTA.
prefill32: the same on 32 experts (2.4 GB of weights; several tiles per SM, so the
         persistent kernel's steady state dominates rather than its tail).
block<T>: the whole MoE block (MoEBlock.forward, seeded GLM-5.2 weights) on T tokens.
pairab <per> <reps> [E]: E experts (default 32) with `per` tokens each (balanced layout,
         256-token blocks), the prefill w13+SwiGLU and w2 launches with SM-pair tiles and
         with single-CTA persistent tiles (FUS_GEMM_NO_PAIR), interleaved rep by rep.
         per = "real": seeded counts in 202..311 per expert, the spread of the seeded
         T=8192 routing over 256 experts (about half the experts take two blocks).
Each launch is timed with CUDA events; the line printed gives us and TB/s or TF/s.
"""

from __future__ import annotations

import sys

import torch

from .. import ops, synth


def block_case(T: int, reps: int) -> None:
    from ..block import MoEBlock

    d = synth.Dims()
    w = synth.make_block_weights(1, d, "cuda")
    blk = MoEBlock(w["gamma"], w["gate_w"], w["bias"], w["w13"], w["w2"], w["w13s"], w["w2s"])
    h, r = synth.make_inputs(1000 + T, T, d, "cuda")
    blk(h, r)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(reps + 1)]
    ev[0].record()
    for i in range(reps):
        blk(h, r)
        ev[i + 1].record()
    torch.cuda.synchronize()
    ops.check_status()
    ts = [ev[i].elapsed_time(ev[i + 1]) * 1e3 for i in range(reps)]
    print(f"block T={T}: " + " ".join(f"{t:.0f}" for t in ts) + " us per call")


def pair_ab(per, reps: int, E: int = 32) -> None:
    import numpy as np

    H, I, K = 6144, 2048, 8
    w13 = synth.make("w13", (E, 2 * I, H), 1, "cuda")
    w2 = synth.make("w2", (E, H, I), 1, "cuda")
    bn = 256
    if per == "real":
        rng = np.random.default_rng(8192)
        counts = rng.integers(202, 312, E)
        flat = np.repeat(np.arange(E), counts)
        flat = rng.permutation(flat)[: len(flat) // K * K]
        T = len(flat) // K
        ids = torch.from_numpy(flat.astype(np.int32)).view(T, K).cuda()
    else:
        per = int(per)
        T = per * E // K
        ids = (torch.arange(T * K, device="cuda") % E).view(T, K).to(torch.int32)
    R = T * K
    cap = (R + E * (bn - 1) + bn - 1) // bn * bn
    s = torch.empty(cap, dtype=torch.int32, device="cuda")
    e = torch.empty(cap // bn, dtype=torch.int32, device="cuda")
    n = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.moe_align(ids, E, bn, s, e, n, flags=ops.ALIGN_BALANCED)
    x = synth.make("h", (T, H), 1, "cuda")
    xs = torch.empty(cap, H, dtype=torch.bfloat16, device="cuda")
    ops.permute_rows(x, s, n, K, R, xs, cap)
    act = torch.empty(cap, I, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(cap, H, dtype=torch.bfloat16, device="cuda")
    maxb = min(R, E) + R // bn

    def launch(flag):
        g13 = [ops.gemm_group(w13, xs, act, expert_ids=e, ntp=n, max_blocks=maxb,
                              row_limit=cap, flags=ops.GEMM_SWIGLU_EXACT | flag, live_ids=s,
                              live_limit=R)]
        g2 = [ops.gemm_group(w2, act, y, expert_ids=e, ntp=n, max_blocks=maxb, row_limit=cap,
                             live_ids=s, live_limit=R, flags=flag)]
        return (lambda: ops.grouped_gemm(g13, 2 * I, H, ops.FUS_EPI_SWIGLU, bn),
                lambda: ops.grouped_gemm(g2, H, I, ops.FUS_EPI_BF16, bn))

    variants = {"pair": launch(0), "single": launch(ops.GEMM_NO_PAIR)}
    tim = {}
    for _ in range(reps):
        for nm, (a13, a2) in variants.items():
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record()
            a13()
            ev[1].record()
            a2()
            ev[2].record()
            tim.setdefault(nm, []).append(ev)
    torch.cuda.synchronize()
    ops.check_status()
    f13, f2 = 2 * R * H * 2 * I, 2 * R * I * H
    for nm, v in tim.items():
        t13 = sorted(x[0].elapsed_time(x[1]) for x in v)[len(v) // 2]
        t2 = sorted(x[1].elapsed_time(x[2]) for x in v)[len(v) // 2]
        print(f"per={per} {nm}: w13 {t13 * 1e3:.1f} us {f13 / t13 / 1e9:.0f} TF/s; "
              f"w2 {t2 * 1e3:.1f} us {f2 / t2 / 1e9:.0f} TF/s")


def main(case: str, reps: int = 3) -> None:
    if case.startswith("block"):
        block_case(int(case[5:]), reps)
        return
    H, I, K = 6144, 2048, 8
    E = 32 if case == "prefill32" else 16
    w13 = synth.make("w13", (E, 2 * I, H), 1, "cuda")
    w2 = synth.make("w2", (E, H, I), 1, "cuda")
    w13s = synth.make("w13s", (2 * I, H), 1, "cuda")
    w2s = synth.make("w2s", (H, I), 1, "cuda")
    if case.startswith("prefill"):
        T, bn = 32 * E, 256
        ids = (torch.arange(T * K, device="cuda") % E).view(T, K).to(torch.int32)
    else:
        T, bn = 1, 16
        ids = torch.arange(K, device="cuda", dtype=torch.int32).view(1, K)
    R = T * K
    cap = (R + E * (bn - 1) + bn - 1) // bn * bn
    s = torch.empty(cap, dtype=torch.int32, device="cuda")
    e = torch.empty(cap // bn, dtype=torch.int32, device="cuda")
    n = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.moe_align(ids, E, bn, s, e, n)
    x = synth.make("h", (T, H), 1, "cuda")
    act = torch.empty(cap, I, dtype=torch.bfloat16, device="cuda")
    act_s = torch.empty(T, I, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
    ys = torch.empty(T, H, dtype=torch.float32, device="cuda")
    maxb = min(R, E) + R // bn
    decode = not case.startswith("prefill")
    ws = ops.GEMM_W_STREAM if decode else 0
    if decode:  # rows gathered inside the GEMM, as the decode block does
        g13 = [ops.gemm_group(w13, x, act, expert_ids=e, ntp=n, max_blocks=maxb, row_limit=cap,
                              flags=ops.GEMM_SWIGLU_EXACT | ws, live_ids=s, live_limit=R,
                              gather_ids=s, gather_div=K),
               ops.gemm_group(w13s, x, act_s, max_blocks=1, row_limit=T,
                              flags=ops.GEMM_SWIGLU_EXACT | ws)]
    else:
        xs = torch.empty(cap, H, dtype=torch.bfloat16, device="cuda")
        ops.permute_rows(x, s, n, K, R, xs, cap)
        g13 = [ops.gemm_group(w13, xs, act, expert_ids=e, ntp=n, max_blocks=maxb, row_limit=cap,
                              flags=ops.GEMM_SWIGLU_EXACT, live_ids=s, live_limit=R)]
    if decode:  # rows to pair order (the decode block merges from there)
        g2 = [ops.gemm_group(w2, act, y, expert_ids=e, ntp=n, max_blocks=maxb, row_map=s,
                             row_limit=R, live_ids=s, live_limit=R, flags=ws)]
    else:  # rows stay in dispatch order (dense tile stores), as the prefill block does
        y = torch.empty(cap, H, dtype=torch.bfloat16, device="cuda")
        g2 = [ops.gemm_group(w2, act, y, expert_ids=e, ntp=n, max_blocks=maxb, row_limit=cap,
                             live_ids=s, live_limit=R, flags=ws)]
    if decode:
        g2.append(ops.gemm_group(w2s, act_s, ys, max_blocks=1, row_limit=T,
                                 flags=ops.GEMM_OUT_F32 | ws))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    for _ in range(reps):
        ev[0].record()
        ops.grouped_gemm(g13, 2 * I, H, ops.FUS_EPI_SWIGLU, bn)
        ev[1].record()
        ops.grouped_gemm(g2, H, I, ops.FUS_EPI_BF16, bn)
        ev[2].record()
    torch.cuda.synchronize()
    ops.check_status()
    t13, t2 = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    ne = (K + 1) if decode else E
    b13, b2 = ne * 2 * I * H * 2, ne * H * I * 2
    f13, f2 = 2 * (R + (T if decode else 0)) * H * 2 * I, 2 * (R + (T if decode else 0)) * I * H
    print(f"{case}: w13 {t13 * 1e3:.1f} us ({b13 / t13 / 1e9:.2f} TB/s weights, "
          f"{f13 / t13 / 1e9:.1f} TF/s); w2 {t2 * 1e3:.1f} us ({b2 / t2 / 1e9:.2f} TB/s, "
          f"{f2 / t2 / 1e9:.1f} TF/s)")


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "pairab":
        pair_ab(sys.argv[2], int(sys.argv[3]), int(sys.argv[4]) if len(sys.argv) > 4 else 32)
    else:
        main(sys.argv[1] if len(sys.argv) > 1 else "decode",
             int(sys.argv[2]) if len(sys.argv) > 2 else 3)
