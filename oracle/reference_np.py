"""CPU oracle for the GLM-5.2 MoE block — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's torch path, glm52_h200/reference.py (frozen
arithmetic shared with glm52/reference.py). Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference arm may import this module, and only as
the checker; the product (``fusion_b200``) never calls it.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against
golden vectors produced by importing the reference itself (``tests/golden/make_golden.py``).

bf16 tensors are carried as float32 arrays whose values are exactly bf16 (every
``to(bf16)`` of the reference is an explicit :func:`bf16` round-to-nearest-even here).
"""

from __future__ import annotations

import numpy as np

RMS_NORM_EPS = 1e-5          # glm52/config.py:44
TOPK = 8                     # glm52/config.py:24
ROUTED_SCALING_FACTOR = 2.5  # glm52/config.py:25
NORM_TOPK_PROB = True        # glm52/config.py:26


def bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bf16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(a.shape)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------------
# Norms / activations  (glm52_h200/reference.py:57-78)
# ---------------------------------------------------------------------------------
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float = RMS_NORM_EPS) -> np.ndarray:
    """reference.py:57-62: bf16((x*rstd).to(bf16) * w); the mid rounding is deliberate."""
    xf = x.astype(np.float32)
    rstd = (1.0 / np.sqrt((xf * xf).mean(-1, keepdims=True, dtype=np.float32) + np.float32(eps))
            ).astype(np.float32)
    return bf16(bf16(xf * rstd) * w)


def add_rmsnorm(x, residual, w, eps: float = RMS_NORM_EPS):
    """reference.py:65-70: returns (normed, new_residual)."""
    h = bf16(x.astype(np.float32) + residual.astype(np.float32))
    return rmsnorm(h, w, eps), h


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (np.float32(1.0) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def silu_and_mul(x: np.ndarray) -> np.ndarray:
    """reference.py:73-77: [gate | up] -> bf16(silu(gate) * up)."""
    d = x.shape[-1] // 2
    return bf16(silu(x[..., :d].astype(np.float32)) * x[..., d:].astype(np.float32))


def silu_and_mul_exact_fp32(x: np.ndarray) -> np.ndarray:
    """reference.py:113-120 (fp32, no rounding)."""
    d = x.shape[-1] // 2
    xf = x.astype(np.float32)
    return silu(xf[..., :d]) * xf[..., d:]


# ---------------------------------------------------------------------------------
# Router  (reference.py:138-175)
# ---------------------------------------------------------------------------------
def router_logits(x: np.ndarray, gate_w: np.ndarray) -> np.ndarray:
    """reference.py:155: F.linear(x.float(), gate_w.float())."""
    return (x.astype(np.float32) @ gate_w.astype(np.float32).T).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def topk_desc(choice: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest per row, descending; ties -> lower index first."""
    order = np.argsort(-choice, axis=-1, kind="stable")
    return order[..., :k]


def router_select(logits: np.ndarray, correction_bias=None, topk: int = TOPK,
                  n_group: int = 1, topk_group: int = 1, norm_topk_prob: bool = NORM_TOPK_PROB,
                  routed_scaling_factor: float = ROUTED_SCALING_FACTOR):
    """reference.py:156-175 after the logits: sigmoid, +bias for the choice only,
    (grouped) top-k, gather the *unbiased* scores, renormalise, scale."""
    scores = sigmoid(logits)
    choice = scores if correction_bias is None else (scores + correction_bias).astype(np.float32)
    if n_group > 1:
        T, E = choice.shape
        g = choice.reshape(T, n_group, E // n_group)
        top2 = np.sort(g, axis=-1)[..., -2:]
        gscore = top2.sum(-1)
        keep = topk_desc(gscore, topk_group)
        mask = np.zeros_like(gscore)
        np.put_along_axis(mask, keep, 1.0, axis=1)
        choice = (g * mask[..., None]).reshape(T, E)
    ids = topk_desc(choice, topk)
    w = np.take_along_axis(scores, ids, axis=1).astype(np.float32)
    if norm_topk_prob:
        s = w.sum(-1, keepdims=True, dtype=np.float32)
        w = (w / np.maximum(s, np.float32(1e-20))).astype(np.float32)
    w = (w * np.float32(routed_scaling_factor)).astype(np.float32)
    return w, ids.astype(np.int32)


def router(x, gate_w, correction_bias=None, **kw):
    logits = router_logits(x, gate_w)
    w, ids = router_select(logits, correction_bias, **kw)
    return logits, w, ids


# ---------------------------------------------------------------------------------
# Dispatch layout  (reference.py:179-222, sglang moe_align_block_size)
# ---------------------------------------------------------------------------------
def moe_align_block_size(topk_ids: np.ndarray, block_m: int, num_experts: int):
    flat = topk_ids.reshape(-1).astype(np.int64)
    numel = flat.size
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=num_experts)
    padded = (counts + block_m - 1) // block_m * block_m
    total = int(padded.sum())
    sorted_token_ids = np.full(total, numel, dtype=np.int32)
    expert_ids = np.zeros(total // block_m, dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(padded)[:-1]]).astype(np.int64)
    src = 0
    for e in range(num_experts):
        c, s = int(counts[e]), int(starts[e])
        if c:
            sorted_token_ids[s:s + c] = order[src:src + c]
            src += c
        nblk = int(padded[e]) // block_m
        if nblk:
            expert_ids[s // block_m: s // block_m + nblk] = e
    return sorted_token_ids, expert_ids, np.array([total], dtype=np.int32)


# ---------------------------------------------------------------------------------
# Expert MLPs  (reference.py:228-311)
# ---------------------------------------------------------------------------------
def _linear_bf16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """F.linear at bf16: fp32 accumulation, one rounding of the result."""
    return bf16(x.astype(np.float32) @ w.astype(np.float32).T)


def moe_mlp(x, get_w13, get_w2, topk_weights, topk_ids, num_experts: int) -> np.ndarray:
    """reference.py:228-259 (framework path): per expert, bf16 GEMM -> bf16 SwiGLU ->
    bf16 GEMM, weighted fp32 index_add, bf16 result. ``get_w13(e)`` / ``get_w2(e)``
    return one expert's [2I,H] / [H,I] weights (lets callers materialise only the
    experts that are routed to)."""
    T, H = x.shape
    out = np.zeros((T, H), dtype=np.float32)
    for e in range(num_experts):
        rows, ks = np.nonzero(topk_ids == e)
        if rows.size == 0:
            continue
        h = _linear_bf16(x[rows], get_w13(e))
        a = silu_and_mul(h)
        y = _linear_bf16(a, get_w2(e))
        np.add.at(out, rows, y * topk_weights[rows, ks][:, None])
    return bf16(out)


def moe_mlp_exact_fp32(x, get_w13, get_w2, topk_weights, topk_ids, num_experts: int):
    """reference.py:262-291: no intermediate rounding, fp32 result."""
    T, H = x.shape
    out = np.zeros((T, H), dtype=np.float32)
    for e in range(num_experts):
        rows, ks = np.nonzero(topk_ids == e)
        if rows.size == 0:
            continue
        h = x[rows].astype(np.float32) @ get_w13(e).astype(np.float32).T
        a = silu_and_mul_exact_fp32(h)
        y = a @ get_w2(e).astype(np.float32).T
        np.add.at(out, rows, y * topk_weights[rows, ks][:, None])
    return out


def shared_expert_mlp(x, w13_s, w2_s) -> np.ndarray:
    """reference.py:294-311: fp32 GEMM, bf16 h, framework SwiGLU, fp32 result."""
    h = x.astype(np.float32) @ w13_s.astype(np.float32).T
    a = silu_and_mul(bf16(h))
    return (a @ w2_s.astype(np.float32).T).astype(np.float32)


def expert_merge(per_expert_out: np.ndarray, topk_weights: np.ndarray) -> np.ndarray:
    """reference.py:314-344 (glm52/reference.py:159-188): bf16(sum_k w_k * y_k) over unweighted y [T, k, H]."""
    return bf16((per_expert_out.astype(np.float32) * topk_weights[..., None]).sum(1))


def moe_block(h, r, gamma, gate_w, bias, get_w13, get_w2, w13_s, w2_s, num_experts: int,
              topk: int = TOPK, eps: float = RMS_NORM_EPS):
    """The block as glm52/bench/bench_layer.py:365-374 composes it (no o_proj):
    out = bf16(moe_mlp(x2) + h1 + shared(x2)). Returns a dict of every stage."""
    x2, h1 = add_rmsnorm(h, r, gamma, eps)
    logits, tw, ti = router(x2, gate_w, bias, topk=topk)
    routed = moe_mlp(x2, get_w13, get_w2, tw, ti, num_experts)
    acc = routed + h1
    if w13_s is not None:
        acc = acc + shared_expert_mlp(x2, w13_s, w2_s)
    return {"h1": h1, "x2": x2, "logits": logits, "topk_weights": tw, "topk_ids": ti,
            "routed": routed, "out": bf16(acc)}


def shared_expert_mlp_exact_fp32(x, w13_s, w2_s) -> np.ndarray:
    """shared_expert_mlp (reference.py:294-311) without its one bf16 rounding of h,
    i.e. the exact-fp32 twin built from silu_and_mul_exact_fp32 (reference.py:113-120)."""
    h = x.astype(np.float32) @ w13_s.astype(np.float32).T
    return (silu_and_mul_exact_fp32(h) @ w2_s.astype(np.float32).T).astype(np.float32)


def moe_block_exact_fp32(x2, h1, topk_weights, topk_ids, get_w13, get_w2, w13_s, w2_s,
                         num_experts: int) -> np.ndarray:
    """The block's fp32 path from the reference's exact functions: routed experts via
    moe_mlp_exact_fp32 (reference.py:262-291) + h1 + the exact shared expert, never
    rounded (x2 / h1 stay the bf16 tensors the block must store). Returns fp32."""
    acc = moe_mlp_exact_fp32(x2, get_w13, get_w2, topk_weights, topk_ids, num_experts)
    acc = acc + h1.astype(np.float32)
    if w13_s is not None:
        acc = acc + shared_expert_mlp_exact_fp32(x2, w13_s, w2_s)
    return acc.astype(np.float32)


# ---------------------------------------------------------------------------------
# o_proj + ResAdd1  (glm52/bench/bench_layer.py:355; glm52/kernels/oproj_resadd.py)
# ---------------------------------------------------------------------------------
def oproj_resadd(a: np.ndarray, w_kn: np.ndarray, residual, fused: bool = True) -> np.ndarray:
    """h1 for attention output a [T, K] and o_proj weight w_kn [K, N] (bf16 values):
    fused (bench_layer.py:355, oproj_resadd.py FUSE_RESADD): bf16(a @ w + residual) in fp32;
    unfused without split-K (oproj_resadd.py:216-221): c = bf16(a @ w), h1 = bf16(c + residual)."""
    acc = a.astype(np.float32) @ w_kn.astype(np.float32)
    if not fused:
        acc = bf16(acc)
    if residual is not None:
        acc = acc + residual.astype(np.float32)
    return bf16(acc)


# ---------------------------------------------------------------------------------
# Lazy pre-norm, half fused  (glm52/kernels/lazy_prenorm.py; exact form reference.py:123)
# ---------------------------------------------------------------------------------
def row_rstd(x: np.ndarray, eps: float = RMS_NORM_EPS) -> np.ndarray:
    """lazy_prenorm.py:347 rstd_kernel: 1/sqrt(mean(x^2) + eps) in fp32 per row."""
    xf = x.astype(np.float32)
    return (np.float32(1.0) / np.sqrt((xf * xf).mean(-1, dtype=np.float32) + np.float32(eps))
            ).astype(np.float32)


def fold_weight_rowmajor(b_kn: np.ndarray, w: np.ndarray) -> np.ndarray:
    """lazy_prenorm.py:75: B [K, N], row k scaled by w[k], rounded to bf16."""
    return bf16(b_kn.astype(np.float32) * w.astype(np.float32)[:, None])


def fold_weight_nk(bt: np.ndarray, w: np.ndarray) -> np.ndarray:
    """lazy_prenorm.py:80: B^T [..., N, K], column k scaled by w[k], rounded to bf16."""
    return bf16(bt.astype(np.float32) * w.astype(np.float32))


def lazy_router_logits(h: np.ndarray, b_folded_kn: np.ndarray, eps: float = RMS_NORM_EPS):
    """The F11b' router: (h @ B_folded) * rstd(h), fp32."""
    return ((h.astype(np.float32) @ b_folded_kn.astype(np.float32)) *
            row_rstd(h, eps)[:, None]).astype(np.float32)


def router_logits_exact_fp32(h: np.ndarray, w: np.ndarray, gate_w: np.ndarray,
                             eps: float = RMS_NORM_EPS) -> np.ndarray:
    """reference.py:123-132: (h * rstd * w) @ gate_w.T entirely in fp32."""
    hf = h.astype(np.float32)
    xn = hf * row_rstd(h, eps)[:, None] * w.astype(np.float32)
    return (xn @ gate_w.astype(np.float32).T).astype(np.float32)


# ---------------------------------------------------------------------------------
# FP8 checkpoint ingest  (no reference counterpart: FP8 is out of scope there,
# glm52_h200/README.md:194; the format is the e4m3 + per-128x128-block scale of
# block-quantised MoE checkpoints)
# ---------------------------------------------------------------------------------
def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    """OCP FP8 E4M3 (fn variant: no infinities, S.1111.111 = NaN) decoded from its bits."""
    b = bits.astype(np.uint32)
    sign = np.where(b >> 7, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    man = (b & 7).astype(np.float64)
    val = np.where(exp == 0, man / 8.0 * 2.0 ** -6, (1.0 + man / 8.0) * 2.0 ** (exp.astype(np.float64) - 7))
    val = np.where((exp == 15) & ((b & 7) == 7), np.nan, val)
    return (sign * val).astype(np.float32)


def fp8_block_dequant(bits: np.ndarray, scale: np.ndarray, block=(128, 128)) -> np.ndarray:
    """bf16(e4m3(bits) * scale[r // br, c // bc]) (fp32 product, one rounding)."""
    br, bc = block
    R, C = bits.shape
    s = np.repeat(np.repeat(scale.astype(np.float32), br, 0), bc, 1)[:R, :C]
    return bf16(e4m3_to_f32(bits) * s)
