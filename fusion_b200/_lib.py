"""ctypes binding of ``libfusion_b200.so`` (the C ABI in ``include/fusion_b200.h``).

The product path has no fallback: if the library is missing or fails to load, every
call raises. Build it with ``python -m fusion_b200.build``.
"""

from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfusion_b200.so"

vp, i32, i64, f32, sz, u64 = C.c_void_p, C.c_int, C.c_long, C.c_float, C.c_size_t, C.c_ulonglong


class GemmGroup(C.Structure):
    """Mirror of ``fus_gemm_group``."""

    _fields_ = [
        ("w", vp),
        ("n_experts", i32),
        ("x", vp),
        ("ldx", i64),
        ("x_rows", i32),
        ("expert_ids", vp),
        ("ntp", vp),
        ("max_blocks", i32),
        ("out", vp),
        ("ldo", i64),
        ("row_map", vp),
        ("row_limit", i32),
        ("row_scale", vp),
        ("flags", i32),
        ("live_ids", vp),
        ("live_limit", i32),
        ("token_div", i32),
        ("gather_ids", vp),
        ("gather_div", i32),
        ("res", vp),
        ("ldr", i64),
    ]


class MergeSpec(C.Structure):
    """Mirror of ``fus_merge_spec``."""

    _fields_ = [
        ("counters", vp),
        ("parts", i32),
        ("y", vp),
        ("ld_t", i64),
        ("ld_k", i64),
        ("topk", i32),
        ("w", vp),
        ("ldw", i64),
        ("res", vp),
        ("ldr", i64),
        ("extra", vp),
        ("lde", i64),
        ("out", vp),
        ("ldo", i64),
    ]




class BlockDesc(C.Structure):
    """Mirror of ``fus_moe_block_desc``."""

    _fields_ = [
        ("H", i32),
        ("I", i32),
        ("E", i32),
        ("topk", i32),
        ("eps", f32),
        ("routed_scale", f32),
        ("renorm", i32),
        ("gamma", vp),
        ("wa", vp),
        ("nplanes", i32),
        ("bias", vp),
        ("w13", vp),
        ("w2", vp),
        ("w13s", vp),
        ("w2s", vp),
        ("n_group", i32),
        ("topk_group", i32),
        ("flags", i32),
    ]


class EPP2PDesc(C.Structure):
    """Mirror of ``fus_ep_p2p_desc``."""

    _fields_ = [
        ("blk", C.POINTER(BlockDesc)),
        ("E_loc", i32),
        ("W", i32),
        ("rank", i32),
        ("S", i32),
        ("peer_rows", vp),
        ("peer_leid", vp),
        ("peer_dflags", vp),
        ("peer_ret", vp),
        ("peer_cflags", vp),
        ("recv_rows", vp),
        ("recv_leid", vp),
        ("ret_rows", vp),
        ("dflags", vp),
        ("cflags", vp),
        ("epoch", vp),
    ]


# name -> (restype, argtypes). Every symbol of include/fusion_b200.h appears here.
SIGNATURES: dict[str, tuple] = {
    "fus_version": (i32, []),
    "fus_last_error": (C.c_char_p, []),
    "fus_num_sms": (i32, []),
    "fus_add_rmsnorm": (i32, [vp, i64, vp, i64, vp, vp, i64, vp, i64, i32, i32, f32, i32, i32, vp, vp]),
    "fus_router_split_weight": (i32, [vp, vp, i32, i32, vp]),
    "fus_router_transpose_weight": (i32, [vp, vp, i32, i32, vp]),
    "fus_router_nsplit": (i32, [i32, i32, i32, i32]),
    "fus_router_logits": (i32, [vp, i64, vp, i32, vp, i32, i32, i32, i32, vp, vp]),
    "fus_router_topk": (i32, [vp, i32, vp, vp, vp, vp, i32, i32, i32, f32, i32, vp, vp]),
    "fus_router_topk_grouped": (i32, [vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, i32, vp,
                                      vp]),
    "fus_moe_align_workspace": (sz, [i32, i32]),
    "fus_moe_align": (i32, [vp, i32, i32, i32, vp, i32, vp, i32, vp, vp, sz, vp, vp]),
    "fus_moe_align_ex": (i32, [vp, i32, i32, i32, vp, i32, vp, i32, vp, vp, i32, vp, sz, vp, vp]),
    "fus_moe_align_noalloc": (i32, [vp, i32, i32, i32, vp, i32, vp, i32, vp, vp, vp]),
    "fus_moe_route_small": (i32, [vp, vp, vp, f32, vp, i32, vp, i32, i32, i32, i32, f32, i32, vp, vp,
                                  vp, vp, vp, i32, vp, i32, vp, i32, vp, vp, vp, i32, vp, vp]),
    "fus_permute_rows": (i32, [vp, i64, vp, vp, i32, i32, vp, i64, i32, i32, vp, vp]),
    "fus_merge_pos": (i32, [vp, i64, vp, i32, vp, i64, vp, i64, vp, i64, i32, vp, i64, i32, i32,
                            vp, vp]),
    "fus_grouped_gemm": (i32, [C.POINTER(GemmGroup), i32, i32, i32, i32, i32, i32, i32, i64, vp, vp]),
    "fus_grouped_gemm_ex": (i32, [C.POINTER(GemmGroup), i32, i32, i32, i32, i32, i32, i32, i64, i32,
                                  vp, vp]),
    "fus_grouped_gemm_tiles": (i32, [i32, i32, i32]),
    "fus_grouped_gemm_merge": (i32, [C.POINTER(GemmGroup), i32, i32, i32, i32, C.POINTER(MergeSpec),
                                     vp, vp]),
    "fus_silu_and_mul": (i32, [vp, i64, vp, i64, i32, i32, vp, vp]),
    "fus_merge": (i32, [vp, i64, i64, i32, vp, i64, vp, i64, vp, i64, i32, vp, i64, i32, i32, i32, vp,
                        vp]),
    "fus_add": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, vp, vp]),
    "fus_seed": (i32, [vp, i64, vp, i64, i32, i32, i32, vp, vp]),
    "fus_moe_block_pick_block_n": (i32, [i32, i32, i32]),
    "fus_moe_block_workspace": (sz, [C.POINTER(BlockDesc), i32, i32]),
    "fus_moe_block_check": (i32, [C.POINTER(BlockDesc), i32, i32, sz]),
    "fus_moe_block_forward": (
        i32,
        [C.POINTER(BlockDesc), vp, vp, i32, i32, vp, vp, vp, vp, vp, sz, vp, vp],
    ),
    "fus_ep_plan": (i32, [vp, i32, i32, i32, vp, vp, vp, vp, vp]),
    "fus_ep_dispatch_small": (i32, [vp, i64, i32, vp, i32, i32, i32, i32, i32, vp, i64, vp, vp, vp,
                                    vp]),
    "fus_ep_pack": (i32, [vp, i64, i32, vp, i32, i32, vp, vp, i64, vp, vp, vp]),
    "fus_ep_unpack": (i32, [vp, i64, i32, vp, i32, vp, i64, vp, vp]),
    "fus_ep_plan_dedup": (i32, [vp, i32, i32, i32, i32, vp, vp, vp, vp]),
    "fus_ep_pack_dedup": (i32, [vp, i64, i32, vp, i32, i32, vp, vp, i32, i32, vp, vp, vp, i64,
                                vp, vp, vp, vp, i32, vp, vp]),
    "fus_ep_return_rowmap": (i32, [vp, i32, vp, vp, i32, i32, vp, vp, i32, vp, vp, vp]),
    "fus_ep_partial_sum": (i32, [vp, i64, i32, vp, vp, i32, i32, vp, i64, vp, vp]),
    "fus_ipc_handle": (i32, [vp, vp, C.POINTER(C.c_size_t)]),
    "fus_ipc_open": (i32, [vp, sz, C.POINTER(C.c_void_p)]),
    "fus_ipc_close": (i32, [vp, sz]),
    "fus_ep_p2p_dispatch": (i32, [vp, i64, i32, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp,
                                  vp, vp, vp]),
    "fus_ep_p2p_wait": (i32, [vp, vp, i32, u64, vp, vp]),
    "fus_ep_p2p_combine": (i32, [vp, i64, i32, vp, i32, i32, i32, vp, vp, vp, vp, vp]),
    "fus_ep_p2p_decode_workspace": (sz, [vp, i32]),
    "fus_oproj_workspace": (sz, [i32, i32, i32, i32]),
    "fus_oproj_resadd": (i32, [vp, i64, vp, i32, i32, i32, vp, i64, vp, i64, i32, vp, sz, vp, vp]),
    "fus_oproj_f32_workspace": (sz, [i32, i32, i32]),
    "fus_oproj_gemm_f32": (i32, [vp, i64, vp, i32, i32, i32, vp, i64, vp, i64, i32, vp, sz, vp,
                                 vp]),
    "fus_oproj_finish": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, vp, vp]),
    "fus_row_rstd": (i32, [vp, i64, i32, i32, f32, vp, vp, vp]),
    "fus_fp8_block_dequant": (i32, [vp, vp, i64, vp, i64, i32, i32, i32, vp, vp]),
    "fus_fold_weight": (i32, [vp, vp, vp, i64, i32, i32, i64, vp, vp]),
    "fus_scale_sum_planes": (i32, [vp, i32, i64, i32, i32, vp, vp, i64, vp, vp]),
    "fus_ep_p2p_decode_forward": (i32, [vp, vp, vp, i32, vp, vp, vp, vp, vp, sz, vp, vp]),
    "fus_synth_fill": (i32, [vp, i32, i64, i64, u64, f32, f32, vp]),
    "fus_synth_fill_host": (None, [vp, i32, i64, i64, u64, f32, f32]),
}

_lib: C.CDLL | None = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Load the library once; raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH.name} is not built; run `python -m fusion_b200.build` "
                        "(there is no fallback implementation)"
                    )
                h = C.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def last_error() -> str:
    msg = lib().fus_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> int:
    """Call an int-returning entry point; nonzero return -> RuntimeError."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise RuntimeError(f"{name} failed ({rc}): {last_error()}")
    return rc
