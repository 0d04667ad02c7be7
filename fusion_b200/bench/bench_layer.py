"""The layer-chain driver on B200 (drop-in for glm52/bench/bench_layer.py:292-612).

Same structure as the reference: a `LayerProblem` per regime (seeded inputs and GLM-5.2
weights, routing frozen from the pipeline's own x2 with a zero correction bias, an fp32
reference output), `build_chain(p, cfg, sel, shared_cfg)` returning the list of launches
for one fusion configuration, `CONFIGS`, and `main()` which checks every configuration
against the fp32 reference (tol 5e-2, bench_layer.py:573) and times it as one chain with
one L2 flush per repetition. The chain starts at o_proj (S3/S4, bench_layer.py:399-415):
`resadd1="in_oproj"` is fusion #1 (h1 = a_attn @ w_o + h_in in one GEMM, then norm only),
"separate" writes c = a_attn @ w_o and the norm axis adds h_in.

Extra configuration `Z_block`: the whole block as one C-ABI call (fus_moe_block_forward),
which computes its own routing.

    python -m fusion_b200.bench.bench_layer --regimes decode_bs1,prefill_t8192
"""

from __future__ import annotations

import argparse

import torch

from .. import config as C
from .. import synth
from ..block import BlockOutputs, MoEBlock
from ..common import bench_chain, check, record
from ..kernels import add_rmsnorm as KN
from ..kernels import layout as KL
from ..kernels import moe_down_merge as KD
from ..kernels import moe_gateup as KG
from ..kernels import norm_router as KR
from ..kernels import oproj_resadd as KO

H = C.HIDDEN_SIZE
I = C.MOE_INTERMEDIATE_SIZE
E = C.N_ROUTED_EXPERTS
TOPK = C.NUM_EXPERTS_PER_TOK

REGIMES = {
    "decode_bs1": 1,
    "decode_bs32": 32,
    "decode_bs256": 256,
    "decode_bs512": 512,
    "decode_bs1024": 1024,
    "prefill_t2048": 2048,
    "prefill_t8192": 8192,
}


def _bm(rows_per_expert: float) -> int:
    for bm in (16, 32, 64, 128):
        if rows_per_expert <= bm:
            return bm
    return 256


def load_cfgs(regime: str) -> dict:
    """Per-kernel cfg dicts. The only knob the sm_100a kernels take is the dispatch
    block (BLOCK_M = the GEMM's token tile); everything else is fixed by design."""
    T = REGIMES[regime]
    bm = 16 if T * TOPK / E <= 16 else 32 if T * TOPK / E <= 64 else 64 if T * TOPK / E <= 160 else 128
    g = {"BLOCK_M": bm}
    return {"oproj": {}, "add": {}, "norm": {}, "addnorm": {}, "router": {}, "topk": {}, "w13": g,
            "w13_fused": g, "act": {}, "w2": g, "w2_fused8": g, "w2_fused9": g,
            "moe_sum": {}, "resadd2": {}}


class LayerProblem:
    def __init__(self, regime: str, seed: int = 0, weights: dict | None = None):
        T = REGIMES[regime]
        self.regime, self.T, self.rows = regime, T, T * TOPK
        dev, bf = "cuda", torch.bfloat16
        d = synth.Dims()
        w = weights if weights is not None else synth.make_block_weights(seed, d, dev)
        self.weights = w
        # the chain's inputs: attention output `a_attn`, o_proj weight `w_o` [K, H] and the
        # residual `h_in`; c = a_attn @ w_o is the o_proj output of the unfused chain
        self.Kq = C.OPROJ_K_PREFILL if regime.startswith("prefill") else C.OPROJ_K_DECODE
        self.a_attn = synth.make("a_attn", (T, self.Kq), seed * 7919 + T, dev)
        self.w_o = synth.make("w_o", (self.Kq, H), seed + 17, dev)
        self.h_in = synth.make("r", (T, H), seed * 7919 + T, dev)
        self.c = torch.empty(T, H, dtype=bf, device=dev)
        self.acc32 = torch.zeros(T, H, dtype=torch.float32, device=dev)
        self.h1 = torch.empty(T, H, dtype=bf, device=dev)
        self.w_norm = w["gamma"]
        self.x2 = torch.empty(T, H, dtype=bf, device=dev)
        self.wg_t = KR.wgt_from_gate(w["gate_w"].to(bf))  # [H, E] bf16, like the reference
        self.logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        self.topw = torch.empty(T, TOPK, dtype=torch.float32, device=dev)
        self.topi = torch.empty(T, TOPK, dtype=torch.int32, device=dev)
        self.w13, self.w2 = w["w13"], w["w2"]
        self.inter = torch.empty(self.rows, 2 * I, dtype=bf, device=dev)
        self.act = torch.empty(self.rows, I, dtype=bf, device=dev)
        self.y3 = torch.zeros(self.rows, H, dtype=bf, device=dev)
        self.y3v = self.y3.view(T, TOPK, H)
        self.routed = torch.zeros(T, H, dtype=bf, device=dev)
        self.out = torch.zeros(T, H, dtype=bf, device=dev)
        self.w13s, self.w2s = w["w13s"].unsqueeze(0), w["w2s"].unsqueeze(0)
        self.s_inter = torch.empty(T, 2 * I, dtype=bf, device=dev)
        self.s_act = torch.empty(T, I, dtype=bf, device=dev)
        self.s_out = torch.empty(T, H, dtype=bf, device=dev)

        # routing frozen from the pipeline's own x2 (bench_layer.py:348-363), zero bias
        with torch.no_grad():
            KO.gemm_launch(self.a_attn, self.w_o, self.c, None, {}, False, False)
            KN.fused_add_rmsnorm(self.c, self.h_in, self.w_norm, self.h1, self.x2, {})
            KR.router_gemm(self.x2, self.wg_t, self.logits, {})
            KR.topk_only(self.logits, self.topw, self.topi, {})
        self.tw_flat = self.topw.flatten().contiguous()
        self.topw_scratch = torch.empty_like(self.topw)
        self.topi_scratch = torch.empty_like(self.topi)
        self.ref_out = self._reference()
        self._layouts: dict[int, tuple] = {}
        self._shared_layouts: dict[int, tuple] = {}

    def _reference(self) -> torch.Tensor:
        """fp32 torch restatement of the reference's ref_out (bench_layer.py:365-374):
        bf16(moe_mlp(x2) + h1 + shared(x2)) with the framework's rounding."""
        bfr = lambda t: t.to(torch.bfloat16).float()
        xf = self.x2.float()
        out = torch.zeros(self.T, H, device="cuda")
        for e in torch.unique(self.topi).tolist():
            rows, ks = torch.nonzero(self.topi == e, as_tuple=True)
            h = bfr(xf[rows] @ self.w13[e].float().t())
            a = bfr(torch.nn.functional.silu(h[:, :I]) * h[:, I:])
            y = bfr(a @ self.w2[e].float().t())
            out.index_add_(0, rows, y * self.topw[rows, ks][:, None])
        s_h = bfr(xf @ self.w13s[0].float().t())
        s_y = bfr(torch.nn.functional.silu(s_h[:, :I]) * s_h[:, I:]) @ self.w2s[0].float().t()
        return (bfr(out) + self.h1.float() + s_y).to(torch.bfloat16)

    def layout(self, block_m: int):
        if block_m not in self._layouts:
            self._layouts[block_m] = KL.moe_align_block_size(self.topi, block_m, E)
        return self._layouts[block_m]

    def shared_layout(self, block_m: int):
        if block_m not in self._shared_layouts:
            ids = torch.zeros(self.T, 1, dtype=torch.int32, device="cuda")
            self._shared_layouts[block_m] = KL.moe_align_block_size(ids, block_m, 1)
        return self._shared_layouts[block_m]


def build_chain(p: LayerProblem, cfg: dict, sel: dict, shared_cfg: dict) -> list:
    fns = []
    L = cfg
    # ---- o_proj (+ ResAdd1) ----
    if sel.get("resadd1") == "in_oproj":  # fusion #1
        fns += KO.make_fused_chain(p.a_attn, p.w_o, p.h_in, p.h1, p.acc32, L["oproj"])
    else:
        fns += [lambda: KO.gemm_launch(p.a_attn, p.w_o, p.c, None, L["oproj"], False, False)]
    if sel.get("block"):
        blk = shared_cfg["block"]
        outs = BlockOutputs(out=p.out, h1=p.h1, topw=p.topw_scratch, topi=p.topi_scratch)
        return fns + [lambda: blk.forward(p.c, p.h_in, outs)]

    # ---- ResAdd + RMSNorm ----
    if sel.get("resadd1") == "in_oproj":  # the residual is already in h1
        fns += [lambda: KN.norm_only(p.h1, p.w_norm, p.x2, L["norm"])]
    elif sel["norm"] == "fused3":
        fns += [lambda: KN.fused_add_rmsnorm(p.c, p.h_in, p.w_norm, p.h1, p.x2, L["addnorm"])]
    else:
        fns += [lambda: KN.add_only(p.c, p.h_in, p.h1, L["add"]),
                lambda: KN.norm_only(p.h1, p.w_norm, p.x2, L["norm"])]
    # ---- router + top-k (scratch outputs: routing stays frozen) ----
    fns += [lambda: KR.router_gemm(p.x2, p.wg_t, p.logits, L["router"]),
            lambda: KR.topk_only(p.logits, p.topw_scratch, p.topi_scratch, L["topk"])]
    # ---- w13 (+ SwiGLU) ----
    if sel["gateup"] == "fused6":
        gc = L["w13_fused"]
        sti, eid, ntp = p.layout(gc["BLOCK_M"])
        fns += [lambda: KG.launch_gateup(p.x2, p.w13, p.act, sti, eid, ntp, p.rows, TOPK, I, gc,
                                         True)]
    else:
        gc = L["w13"]
        sti, eid, ntp = p.layout(gc["BLOCK_M"])
        fns += [lambda: KG.launch_gateup(p.x2, p.w13, p.inter, sti, eid, ntp, p.rows, TOPK, I, gc,
                                         False),
                lambda: KG.launch_silu_and_mul(p.inter, p.act, L["act"])]
    # ---- w2 + merge + ResAdd2 ----
    d = sel["down"]
    if d in ("atomic8", "atomic9"):
        wc = L["w2_fused8"] if d == "atomic8" else L["w2_fused9"]
        sti2, eid2, ntp2 = p.layout(wc["BLOCK_M"])
        if d == "atomic8":
            fns += [lambda: KD.launch_seed(p.routed, None, {}, False),
                    lambda: KD.launch_down(p.act, p.w2, p.routed, p.tw_flat, sti2, eid2, ntp2,
                                           p.rows, TOPK, wc, True),
                    lambda: KD.launch_resadd(p.routed, p.h1, p.out, L["resadd2"])]
        else:
            fns += [lambda: KD.launch_seed(p.out, p.h1, {}, True),
                    lambda: KD.launch_down(p.act, p.w2, p.out, p.tw_flat, sti2, eid2, ntp2,
                                           p.rows, TOPK, wc, True)]
    else:
        wc = L["w2"]
        sti2, eid2, ntp2 = p.layout(wc["BLOCK_M"])
        fns += [lambda: KD.launch_down(p.act, p.w2, p.y3, p.tw_flat, sti2, eid2, ntp2, p.rows,
                                       TOPK, wc, False)]
        if d == "merge_f10":
            fns += [lambda: KD.launch_moe_sum(p.y3v, p.out, p.h1, TOPK, L["moe_sum"], True)]
        else:
            fns += [lambda: KD.launch_moe_sum(p.y3v, p.routed, p.h1, TOPK, L["moe_sum"], False),
                    lambda: KD.launch_resadd(p.routed, p.h1, p.out, L["resadd2"])]
    # ---- shared expert ----
    sg, sd = shared_cfg["w13"], shared_cfg["w2"]
    ssti, seid, sntp = p.shared_layout(sg["BLOCK_M"])
    ssti2, seid2, sntp2 = p.shared_layout(sd["BLOCK_M"])
    ones = shared_cfg["ones"]
    fns += [
        lambda: KG.launch_gateup(p.x2, p.w13s, p.s_inter, ssti, seid, sntp, p.T, 1, I, sg, False),
        lambda: KG.launch_silu_and_mul(p.s_inter, p.s_act, shared_cfg["act"]),
        lambda: KD.launch_down(p.s_act, p.w2s, p.s_out, ones, ssti2, seid2, sntp2, p.T, 1, sd,
                               False),
        lambda: KD.launch_resadd(p.s_out, p.out, p.out, L["resadd2"]),
    ]
    return fns


def tune_shared(p: LayerProblem) -> dict:
    """The shared expert is one dense expert over T rows: its token tile follows T."""
    bm = _bm(p.T)
    blk = MoEBlock(p.w_norm, p.wg_t.t().contiguous(), torch.zeros(E, device="cuda"),
                   p.w13, p.w2, p.w13s[0], p.w2s[0])
    return {"w13": {"BLOCK_M": bm}, "act": {}, "w2": {"BLOCK_M": bm},
            "ones": torch.ones(p.T, device="cuda"), "block": blk}


CONFIGS = {
    "A_all_unfused": dict(resadd1="separate", norm="split", gateup="split", down="split"),
    "B_f3": dict(resadd1="separate", norm="fused3", gateup="split", down="split"),
    "C_f1": dict(resadd1="in_oproj", norm="split", gateup="split", down="split"),
    "D_f6": dict(resadd1="separate", norm="split", gateup="fused6", down="split"),
    "E_f10": dict(resadd1="separate", norm="split", gateup="split", down="merge_f10"),
    "F_f8": dict(resadd1="separate", norm="split", gateup="split", down="atomic8"),
    "G_f9": dict(resadd1="separate", norm="split", gateup="split", down="atomic9"),
    "H_f3_f10": dict(resadd1="separate", norm="fused3", gateup="split", down="merge_f10"),
    "I_f3_f9": dict(resadd1="separate", norm="fused3", gateup="split", down="atomic9"),
    "J_f1_f6_f9": dict(resadd1="in_oproj", norm="split", gateup="fused6", down="atomic9"),
    "K_f3_f8": dict(resadd1="separate", norm="fused3", gateup="split", down="atomic8"),
    "L_f3_f6_f10": dict(resadd1="separate", norm="fused3", gateup="fused6", down="merge_f10"),
    "Z_block": dict(resadd1="separate", block=True),
}


def run_regime(regime: str, rep: int = 40, weights: dict | None = None, verbose: bool = True):
    p = LayerProblem(regime, weights=weights)
    cfg = load_cfgs(regime)
    shared = tune_shared(p)
    rows = {}
    for name, sel in CONFIGS.items():
        chain = build_chain(p, cfg, sel, shared)
        p.out.zero_(); p.routed.zero_(); p.y3.zero_()
        for fn in chain:
            fn()
        torch.cuda.synchronize()
        ck = check(p.out.clone(), p.ref_out, tol=5e-2, label=name)
        t = bench_chain(chain, warmup=5, rep=rep)
        rows[name] = {"ms": t.p50_ms, "p10_p90": [t.p10_ms, t.p90_ms], "n_kernels": len(chain),
                      "sel": sel, "rel_err_vs_fp32_ref": ck["rel_err"], "correct": ck["ok"]}
        if verbose:
            print(f"  {name:<14} {t.p50_ms:9.4f} ms ({len(chain):2d} launches) "
                  f"relerr {ck['rel_err']:.2e} {'OK' if ck['ok'] else 'FAIL'}", flush=True)
    ok = {k: v for k, v in rows.items() if v["correct"]}
    best = min(ok, key=lambda k: ok[k]["ms"]) if ok else None
    return {"rows": rows, "best": best, "T": p.T, "moe_rows": p.rows}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--regimes", default=",".join(REGIMES))
    ap.add_argument("--rep", type=int, default=40)
    args = ap.parse_args()
    weights = synth.make_block_weights(0, synth.Dims(), "cuda")
    out = {}
    for regime in [r.strip() for r in args.regimes.split(",") if r.strip()]:
        print(f"\n===== {regime} =====", flush=True)
        out[regime] = run_regime(regime, args.rep, weights)
        print(f"  --> BEST {out[regime]['best']}", flush=True)
    record("layer_configurations_b200", {"configs": CONFIGS, "regimes": out})


if __name__ == "__main__":
    main()
