"""Torch-tensor wrappers over the C ABI (device pointers + the current CUDA stream).

PyTorch only supplies device memory and streams here; all arithmetic runs in the
library's sm_100a kernels. Every wrapper is destination-passing like the C ABI and
raises ``RuntimeError`` when the library rejects its arguments.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L

FUS_EPI_BF16, FUS_EPI_SWIGLU, FUS_EPI_F32 = 0, 1, 2
GEMM_OUT_F32, GEMM_SWIGLU_EXACT, GEMM_W_STREAM, GEMM_MERGE, GEMM_NO_PERSIST = 0x1, 0x2, 0x4, 0x8, 0x10
GEMM_NO_PAIR = 0x40
GEMM_PAIR_NARROW = 0x80
GEMM_SCALE_TOKEN = 0x20
ERR_TIMEOUT, ERR_BAD_EXPERT, ERR_CAPACITY = 0x1, 0x2, 0x4

_status: dict[int, torch.Tensor] = {}


_empty_anchor: dict[int, torch.Tensor] = {}


def _p(t: torch.Tensor | None) -> int | None:
    """Device address of `t`. An empty tensor has no storage (address 0); it is passed as
    an aligned dummy address of its device so that a call over zero rows reaches the
    library's empty-size early return instead of its null-pointer check."""
    if t is None:
        return None
    if t.numel() == 0 and t.is_cuda:
        idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
        a = _empty_anchor.get(idx)
        if a is None:
            a = torch.zeros(256, dtype=torch.uint8, device=t.device)
            _empty_anchor[idx] = a
        return a.data_ptr()
    return t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def status_tensor(device: torch.device | int | None = None) -> torch.Tensor:
    """The per-device int32 status word the kernels OR error bits into."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    t = _status.get(dev.index)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _status[dev.index] = t
    return t


def _sp() -> int:
    return status_tensor().data_ptr()


def read_status(clear: bool = True) -> int:
    """Synchronise and return (then clear) the device status bits."""
    t = status_tensor()
    v = int(t.item())
    if clear and v:
        t.zero_()
    return v


def check_status() -> None:
    v = read_status()
    if v:
        names = [n for b, n in ((ERR_TIMEOUT, "timeout"), (ERR_BAD_EXPERT, "bad expert id"),
                                (ERR_CAPACITY, "capacity")) if v & b]
        raise RuntimeError(f"device status {v:#x}: {', '.join(names)}")


def _ld(t: torch.Tensor) -> int:
    assert t.dim() >= 2 and t.stride(-1) == 1, "rows must be contiguous"
    return t.stride(-2)


# -------------------------------------------------------------------------------------
def add_rmsnorm(x, res, w, h1, out, eps: float = 1e-5, do_add: bool = True, do_norm: bool = True):
    T, N = x.shape
    L.call("fus_add_rmsnorm", _p(x), _ld(x), _p(res), _ld(res) if res is not None else 0, _p(w),
           _p(h1), _ld(h1) if h1 is not None else 0, _p(out), _ld(out) if out is not None else 0,
           T, N, eps, int(do_add), int(do_norm), _stream(), _sp())


def router_split_weight(wg: torch.Tensor) -> torch.Tensor:
    """fp32 [E, H] -> bf16 planes [E, 3H] (hi | mid | lo)."""
    E, H = wg.shape
    wa = torch.empty(E, 3 * H, dtype=torch.bfloat16, device=wg.device)
    L.call("fus_router_split_weight", _p(wg.contiguous()), _p(wa), E, H, _stream())
    return wa


def router_transpose_weight(wgt: torch.Tensor) -> torch.Tensor:
    """bf16 [H, E] -> bf16 [E, H]."""
    H, E = wgt.shape
    wa = torch.empty(E, H, dtype=torch.bfloat16, device=wgt.device)
    L.call("fus_router_transpose_weight", _p(wgt.contiguous()), _p(wa), H, E, _stream())
    return wa


def router_nsplit(T: int, H: int, E: int, nplanes: int) -> int:
    return int(L.lib().fus_router_nsplit(T, H, E, nplanes))


def router_logits(x2, wa, nplanes: int, partial, nsplit: int):
    T, H = x2.shape
    E = wa.shape[0]
    L.call("fus_router_logits", _p(x2), _ld(x2), _p(wa), nplanes, _p(partial), T, H, E, nsplit,
           _stream(), _sp())


def router_topk(partial, nsplit: int, bias, logits_out, topw, topi, scale: float = 2.5,
                renorm: bool = True, n_group: int = 1, topk_group: int = 1):
    T, topk = topi.shape
    E = partial.shape[-1]
    if n_group == 1:
        L.call("fus_router_topk", _p(partial), nsplit, _p(bias), _p(logits_out), _p(topw),
               _p(topi), T, E, topk, scale, int(renorm), _stream(), _sp())
    else:
        L.call("fus_router_topk_grouped", _p(partial), nsplit, _p(bias), _p(logits_out),
               _p(topw), _p(topi), T, E, topk, n_group, topk_group, scale, int(renorm),
               _stream(), _sp())


def moe_align_workspace(numel: int, E: int) -> int:
    return int(L.lib().fus_moe_align_workspace(numel, E))


ALIGN_BALANCED = 0x1


def moe_align(ids, E: int, block_m: int, sorted_ids, expert_ids, ntp, workspace=None,
              pos_of=None, flags: int = 0):
    """Dispatch layout; with ``pos_of`` also each pair's dispatch position, with
    ``flags=ALIGN_BALANCED`` each expert's pairs spread evenly over its blocks."""
    flat = ids.reshape(-1)
    assert flat.is_contiguous() and flat.dtype == torch.int32
    need = moe_align_workspace(flat.numel(), E)
    if need and (workspace is None or workspace.numel() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=ids.device)
    if pos_of is None and not flags:
        L.call("fus_moe_align", _p(flat), flat.numel(), E, block_m, _p(sorted_ids),
               sorted_ids.numel(), _p(expert_ids), expert_ids.numel(), _p(ntp),
               _p(workspace) if need else None, need, _stream(), _sp())
    else:
        L.call("fus_moe_align_ex", _p(flat), flat.numel(), E, block_m, _p(sorted_ids),
               sorted_ids.numel(), _p(expert_ids), expert_ids.numel(), _p(ntp), _p(pos_of),
               flags, _p(workspace) if need else None, need, _stream(), _sp())


def route_small(h, r, gamma, wa, nplanes: int, bias, h1, x2, logits, topw, topi, block_m: int,
                sorted_ids, expert_ids, ntp, done, zero=None, eps: float = 1e-5,
                scale: float = 2.5, renorm: bool = True):
    """Decode front end (T <= 16): norm + router + top-k + layout in one launch."""
    T, H = h.shape
    E = logits.shape[1]
    topk = topi.shape[1]
    L.call("fus_moe_route_small", _p(h), _p(r), _p(gamma), eps, _p(wa), nplanes, _p(bias), T, H, E,
           topk, scale, int(renorm), _p(h1), _p(x2), _p(logits), _p(topw), _p(topi), block_m,
           _p(sorted_ids), sorted_ids.numel(), _p(expert_ids), expert_ids.numel(), _p(ntp),
           _p(done), _p(zero), zero.numel() if zero is not None else 0, _stream(), _sp())


def permute_rows(src, sorted_ids, ntp, div: int, num_valid: int, dst, max_rows: int | None = None):
    H = src.shape[1]
    if max_rows is None:
        max_rows = min(dst.shape[0], sorted_ids.numel())
    L.call("fus_permute_rows", _p(src), _ld(src), _p(sorted_ids), _p(ntp), div, num_valid, _p(dst),
           _ld(dst), max_rows, H, _stream(), _sp())


def gemm_group(w, x, out, *, expert_ids=None, ntp=None, max_blocks: int, row_map=None,
               row_limit: int, row_scale=None, x_rows: int | None = None,
               flags: int = 0, live_ids=None, live_limit: int = 0,
               token_div: int = 1, gather_ids=None, gather_div: int = 1,
               res=None) -> L.GemmGroup:
    """Describe one weight stack + token rows for :func:`grouped_gemm`.

    ``w`` is [n_experts, w_rows, K'] (or [w_rows, K'] for one expert) bf16."""
    g = L.GemmGroup()
    g.w = _p(w)
    g.n_experts = w.shape[0] if w.dim() == 3 else 1
    g.x = _p(x)
    g.ldx = _ld(x)
    g.x_rows = x.shape[0] if x_rows is None else x_rows
    g.expert_ids = _p(expert_ids)
    g.ntp = _p(ntp)
    g.max_blocks = max_blocks
    g.out = _p(out)
    g.ldo = _ld(out)
    g.row_map = _p(row_map)
    g.row_limit = row_limit
    g.row_scale = _p(row_scale)
    g.flags = flags
    g.live_ids = _p(live_ids)
    g.live_limit = live_limit
    g.token_div = token_div
    g.gather_ids = _p(gather_ids)
    g.gather_div = gather_div
    g.res = _p(res)
    g.ldr = _ld(res) if res is not None else 0
    return g


def grouped_gemm(groups: list[L.GemmGroup], w_rows: int, K: int, epilogue: int, block_n: int,
                 a_kplanes: int = 1, ksplit: int = 1, split_stride: int = 0,
                 group_blocks: int = 0):
    arr = (L.GemmGroup * len(groups))(*groups)
    L.call("fus_grouped_gemm_ex", arr, len(groups), w_rows, K, a_kplanes, epilogue, block_n,
           ksplit, split_stride, group_blocks, _stream(), _sp())


def gemm_tiles(w_rows: int, epilogue: int, block_n: int) -> int:
    return int(L.lib().fus_grouped_gemm_tiles(w_rows, epilogue, block_n))


def grouped_gemm_merge(groups: list[L.GemmGroup], w_rows: int, K: int, block_n: int, *,
                       counters, y3, w, res, extra, out, parts: int):
    """Down projection with the expert merge fused into its epilogue.
    y3: [T, topk, H] bf16 rows the routed group writes; counters: zeroed int32
    [T * gemm_tiles(w_rows, FUS_EPI_BF16, block_n)] (left zero afterwards)."""
    m = L.MergeSpec()
    m.counters = _p(counters)
    m.parts = parts
    m.y = _p(y3)
    m.ld_t, m.ld_k = y3.stride(0), y3.stride(1)
    m.topk = y3.shape[1]
    m.w = _p(w)
    m.ldw = w.stride(0)
    m.res = _p(res)
    m.ldr = _ld(res) if res is not None else 0
    m.extra = _p(extra)
    m.lde = _ld(extra) if extra is not None else 0
    m.out = _p(out)
    m.ldo = _ld(out)
    arr = (L.GemmGroup * len(groups))(*groups)
    L.call("fus_grouped_gemm_merge", arr, len(groups), w_rows, K, block_n, C.byref(m), _stream(),
           _sp())


def silu_and_mul(x, y):
    M, twoI = x.shape
    L.call("fus_silu_and_mul", _p(x), _ld(x), _p(y), _ld(y), M, twoI // 2, _stream(), _sp())


def merge(y3, w, res, extra, out, round_mid: bool = True):
    """y3: [T, K, H] view (unit stride along H); extra: bf16 or fp32 [T, H]."""
    T, K, H = y3.shape
    L.call("fus_merge", _p(y3), y3.stride(0), y3.stride(1), K, _p(w),
           w.stride(0) if w is not None else 0, _p(res), _ld(res) if res is not None else 0,
           _p(extra), _ld(extra) if extra is not None else 0,
           int(extra is not None and extra.dtype == torch.float32), _p(out), _ld(out), T, H,
           int(round_mid), _stream(), _sp())


def merge_pos(y, pos_of, K: int, w, res, extra, out):
    """merge over rows in dispatch order: row (t, k) = y[pos_of[t*K + k]] (y: [rows, H])."""
    T, H = out.shape
    L.call("fus_merge_pos", _p(y), _ld(y), _p(pos_of), K, _p(w),
           w.stride(0) if w is not None else 0, _p(res), _ld(res) if res is not None else 0,
           _p(extra), _ld(extra) if extra is not None else 0,
           int(extra is not None and extra.dtype == torch.float32), _p(out), _ld(out), T, H,
           _stream(), _sp())


def oproj_resadd(a, w_nk, res, out, fuse: bool = True, workspace=None):
    """out = bf16(a @ w_nk.T + res) (fuse) or bf16(bf16(a @ w_nk.T) + res); w_nk is the
    K-major [N, K] weight."""
    T, K = a.shape
    N = w_nk.shape[0]
    need = int(L.lib().fus_oproj_workspace(T, N, K, int(fuse)))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
    L.call("fus_oproj_resadd", _p(a), _ld(a), _p(w_nk), T, N, K, _p(res),
           _ld(res) if res is not None else 0, _p(out), _ld(out), int(fuse), _p(workspace),
           need, _stream(), _sp())


def row_rstd(x, rstd, eps: float = 1e-5):
    T, N = x.shape
    L.call("fus_row_rstd", _p(x), _ld(x), T, N, eps, _p(rstd), _stream(), _sp())


def fold_weight(src, w, dst, by_row: bool):
    """dst = bf16(src * w) along K: rows of a [K, N] weight (by_row) or the last dim."""
    if not (src.dtype == w.dtype == dst.dtype == torch.bfloat16):
        raise TypeError("fold_weight: bf16 weight, norm weight and output required")
    assert src.is_contiguous() and dst.is_contiguous()
    cols = src.shape[-1]
    rows = src.numel() // cols
    L.call("fus_fold_weight", _p(src), _p(w), _p(dst), rows, cols, int(by_row),
           src.shape[0] if by_row else 1, _stream(), _sp())


def scale_sum_planes(partial, nsplit: int, row_scale, out):
    T, N = out.shape
    L.call("fus_scale_sum_planes", _p(partial), nsplit, T * N, T, N, _p(row_scale), _p(out),
           _ld(out), _stream(), _sp())


def fp8_block_dequant(src, scale, dst, block=(128, 128)):
    """dst (bf16, rows x cols) = fp8 e4m3 src * scale per block (scale [ceil(R/br),
    ceil(C/bc)] fp32)."""
    if src.dtype != torch.float8_e4m3fn or dst.dtype != torch.bfloat16:
        raise TypeError("fp8_block_dequant: e4m3 source and bf16 destination required")
    cols = src.shape[-1]
    rows = src.numel() // cols
    sc = scale.reshape(-1, scale.shape[-1])
    L.call("fus_fp8_block_dequant", _p(src), _p(sc), sc.stride(0), _p(dst), rows, cols,
           block[0], block[1], _stream(), _sp())


def add(a, b, o):
    M, N = a.shape
    L.call("fus_add", _p(a), _ld(a), _p(b), _ld(b), _p(o), _ld(o), M, N, _stream(), _sp())


def seed(o, src=None):
    M, N = o.shape
    L.call("fus_seed", _p(o), _ld(o), _p(src), _ld(src) if src is not None else 0, M, N,
           int(src is not None), _stream(), _sp())


# -------------------------------------------------------------------------------------
def ep_plan(topi, E_loc: int, W: int, dest, leid, counts):
    flat = topi.reshape(-1)
    L.call("fus_ep_plan", _p(flat), flat.numel(), E_loc, W, _p(dest), _p(leid), _p(counts),
           _stream(), _sp())


def ep_dispatch_small(x, topi, E_loc: int, W: int, S: int, rows, leid_out, slot_of_pair):
    T, K = topi.shape
    L.call("fus_ep_dispatch_small", _p(x), _ld(x), x.shape[1], _p(topi), T, K, E_loc, W, S,
           _p(rows), _ld(rows), _p(leid_out), _p(slot_of_pair), _stream(), _sp())


def ep_pack(x, send_ids, n: int, div: int, leid, rows, leid_out):
    L.call("fus_ep_pack", _p(x), _ld(x), x.shape[1], _p(send_ids), n, div, _p(leid), _p(rows),
           _ld(rows), _p(leid_out), _stream(), _sp())


def ep_unpack(rows, send_ids, n: int, y):
    L.call("fus_ep_unpack", _p(rows), _ld(rows), rows.shape[1], _p(send_ids), n, _p(y), _ld(y),
           _stream(), _sp())


def ep_plan_dedup(topi, E_loc: int, W: int, keys, counts):
    """keys[t*W + d] = d if token t has an expert on rank d else -1; counts[d] = rows and
    counts[W + d] = (token, slot) pairs for rank d."""
    T, K = topi.shape
    L.call("fus_ep_plan_dedup", _p(topi), T, K, E_loc, W, _p(keys), _p(counts), _stream(), _sp())


def ep_pack_dedup(x, send_ids, n: int, W: int, topi, topw, E_loc: int, rows, leid_out,
                  pair_pos=None, counts=None, ret_out=None, w_out=None, pos=None,
                  zero_row: int = 0):
    """One row per (token, destination) with its K slots' local expert (-1 off that
    destination); with ret_out, each slot's place in the owner's return rows; with w_out /
    pos, the partial-sum combine's slot weights and merge positions."""
    K = topi.shape[1]
    L.call("fus_ep_pack_dedup", _p(x), _ld(x), x.shape[1], _p(send_ids), n, W, _p(topi),
           _p(topw), K, E_loc, _p(pair_pos), _p(counts), _p(rows), _ld(rows), _p(leid_out),
           _p(ret_out), _p(w_out), _p(pos), zero_row, _stream(), _sp())


def ep_return_rowmap(sorted_ids, ret_idx, K: int, row_prefix, pair_prefix, rowmap, ntp=None):
    """Owner's w2 row map into the return buffer (see fus_ep_return_rowmap); ``ntp``: the
    layout's padded total (entries of sorted_ids past it are not read)."""
    n = ret_idx.numel() // K
    W = row_prefix.numel() - 1
    L.call("fus_ep_return_rowmap", _p(sorted_ids), sorted_ids.numel(), _p(ntp), _p(ret_idx), n, K,
           _p(row_prefix), _p(pair_prefix), W, _p(rowmap), _stream(), _sp())


def ep_partial_sum(y, leid, w, out):
    """out[i] = bf16(sum_j w[i, j] * y[i*K + j] over slots with leid[i, j] >= 0)."""
    n, K = leid.shape
    L.call("fus_ep_partial_sum", _p(y), _ld(y), y.shape[1], _p(leid), _p(w), n, K, _p(out),
           _ld(out), _stream(), _sp())


# -------------------------------------------------------------------------------------
# NVLink peer-memory exchange (CUDA IPC)
def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """CUDA IPC handle (64 bytes) of the allocation holding ``t`` and t's offset in it."""
    h = (C.c_char * 64)()
    off = C.c_size_t(0)
    L.call("fus_ipc_handle", _p(t), C.cast(h, C.c_void_p), C.byref(off))
    return bytes(h), int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Map a peer's exported allocation; returns the device address of its offset."""
    h = (C.c_char * 64).from_buffer_copy(handle)
    ptr = C.c_void_p(0)
    L.call("fus_ipc_open", C.cast(h, C.c_void_p), offset, C.byref(ptr))
    return int(ptr.value)


def ipc_close(ptr: int, offset: int):
    L.call("fus_ipc_close", ptr, offset)


def ep_p2p_dispatch(x, topi, E_loc: int, W: int, S: int, rank: int, peer_rows, peer_leid,
                    peer_flags, epoch, slot_of_pair):
    T, K = topi.shape
    L.call("fus_ep_p2p_dispatch", _p(x), _ld(x), x.shape[1], _p(topi), T, K, E_loc, W, S, rank,
           _p(peer_rows), _p(peer_leid), _p(peer_flags), _p(epoch), _p(slot_of_pair),
           _stream(), _sp())


def ep_p2p_wait(flags, epoch, W: int, timeout_ns: int = 0):
    L.call("fus_ep_p2p_wait", _p(flags), _p(epoch), W, timeout_ns, _stream(), _sp())


def ep_p2p_combine(y, recv_leid, W: int, S: int, rank: int, peer_ret, peer_cflags, epoch):
    L.call("fus_ep_p2p_combine", _p(y), _ld(y), y.shape[1], _p(recv_leid), W, S, rank,
           _p(peer_ret), _p(peer_cflags), _p(epoch), _stream(), _sp())


# -------------------------------------------------------------------------------------
def synth_fill(t: torch.Tensor, seed: int, mean: float = 0.0, std: float = 1.0, offset: int = 0):
    """Fill ``t`` (bf16 or fp32, contiguous) with the seeded synthetic stream."""
    assert t.is_contiguous()
    dtype = {torch.bfloat16: 0, torch.float32: 1}[t.dtype]
    if t.is_cuda:
        L.call("fus_synth_fill", _p(t), dtype, t.numel(), offset, seed, mean, std, _stream())
    else:
        L.lib().fus_synth_fill_host(C.c_void_p(t.data_ptr()), dtype, t.numel(), offset, seed,
                                    mean, std)
    return t
