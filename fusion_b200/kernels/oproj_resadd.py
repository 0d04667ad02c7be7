"""Fusion #1 — o_proj GEMM + residual add (drop-in for glm52/kernels/oproj_resadd.py).

    gemm_launch(a, b, c, r, cfg, fuse_resadd, atomic_out)      (oproj_resadd.py:144)
        c = a @ b (+ r)         bf16 c: one rounding (fused) / the plain GEMM (unfused)
                                fp32 c (atomic_out): c += a @ b (+ r), the split-K acc32
    epilogue_launch(c, r, o, cfg, has_res)                      (oproj_resadd.py:181)
        o = cast(c (+ r))
    make_fused_chain / make_unfused_chain                       (oproj_resadd.py:199/216)

`b` is the reference's [K, N] weight; the tcgen05 GEMM wants it K-major ([N, K]), so a
row-major b is transposed once per weight version (like the reference's load-time
`wgt_from_gate`) and a b that is already the transpose of a K-major weight is used as
is. The Triton mapping keys of `cfg` (BLOCK_*, SPLIT_K, num_warps ...) do not apply.
"""

from __future__ import annotations

import torch

from .. import _lib as L
from .. import ops
from . import _ws


def _w_nk(b: torch.Tensor) -> torch.Tensor:
    """K-major [N, K] bf16 view of the reference's [K, N] weight."""
    bt = b.t()
    if bt.is_contiguous():
        return bt
    return _ws.converted(b, "oproj_nk", lambda: ops.router_transpose_weight(b))


def gemm_launch(a, b, c, r, cfg, fuse_resadd: bool, atomic_out: bool):
    w = _w_nk(b)
    res = r if fuse_resadd else None
    if atomic_out:  # c is the fp32 split-K accumulator: c += a @ b (+ r)
        T, K = a.shape
        N = w.shape[0]
        need = int(L.lib().fus_oproj_f32_workspace(T, N, K))
        ws = _ws.scratch("oproj_f32_ws", need, torch.uint8, a.device)
        L.call("fus_oproj_gemm_f32", ops._p(a), ops._ld(a), ops._p(w), T, N, K, ops._p(res),
               ops._ld(res) if res is not None else 0, ops._p(c), ops._ld(c), 1, ops._p(ws),
               need, ops._stream(), ops._sp())
        return
    T, K = a.shape
    need = int(L.lib().fus_oproj_workspace(T, w.shape[0], K, 1))
    ops.oproj_resadd(a, w, res, c, fuse=True,
                     workspace=_ws.scratch("oproj_ws", need, torch.uint8, a.device))


def epilogue_launch(c, r, o, cfg, has_res: bool):
    res = r if has_res else None
    if c.dtype == torch.float32:
        T, N = o.shape
        L.call("fus_oproj_finish", ops._p(c), ops._ld(c), ops._p(res),
               ops._ld(res) if res is not None else 0, ops._p(o), ops._ld(o), T, N,
               ops._stream(), ops._sp())
    elif res is not None:
        ops.add(c, res, o)
    else:
        ops.seed(o, c)


def make_fused_chain(a, b, r, out, acc32, cfg):
    """FUSED: h1 = bf16(A@B + residual) in one library call (decode splits K into fp32
    planes summed in fixed order instead of the reference's atomics)."""
    return [lambda: gemm_launch(a, b, out, r, cfg, True, False)]


def make_unfused_chain(a, b, r, out, cmat, acc32, gcfg, ecfg):
    """UNFUSED: c materialised, then h1 = c + r. With SPLIT_K > 1 the reference keeps c
    in the fp32 acc32 (one rounding); without it c is bf16 (two roundings)."""
    if (gcfg or {}).get("SPLIT_K", 1) > 1:
        return [
            lambda: acc32.zero_(),
            lambda: gemm_launch(a, b, acc32, None, gcfg, False, True),
            lambda: epilogue_launch(acc32, r, out, ecfg, True),
        ]
    return [
        lambda: gemm_launch(a, b, cmat, None, gcfg, False, False),
        lambda: epilogue_launch(cmat, r, out, ecfg, True),
    ]
