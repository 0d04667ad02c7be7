"""GPU parity: dispatch layout (moe_align) bit-exact against the reference's golden
vectors and the oracle; row permutation."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from fusion_b200 import ops
from gpu_util import DEV, finish
from oracle import reference_np as O

pytestmark = pytest.mark.gpu


def run_align(ids: np.ndarray, bm: int, E: int = 256):
    t = torch.from_numpy(np.ascontiguousarray(ids, dtype=np.int32)).to(DEV)
    n = t.numel()
    cap = n + E * (bm - 1)
    cap = (cap + bm - 1) // bm * bm
    s = torch.full((cap,), -7, dtype=torch.int32, device=DEV)
    e = torch.full((cap // bm,), -7, dtype=torch.int32, device=DEV)
    ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_align(t, E, bm, s, e, ntp)
    finish()
    total = int(ntp.item())
    return s[:total].cpu().numpy(), e[: total // bm].cpu().numpy(), total


def test_align_golden_bit_exact():
    g = golden("align")
    names = sorted({k.rsplit("_", 1)[0] for k in g if k.endswith("_ids")})
    for n in names:
        s, e, total = run_align(g[f"{n}_ids"], int(g[f"{n}_bm"]))
        assert total == int(g[f"{n}_ntp"][0]), n
        assert np.array_equal(s, g[f"{n}_sorted"]), n
        assert np.array_equal(e, g[f"{n}_eids"]), n


@pytest.mark.parametrize("T,bm", [(1024, 16), (1025, 32), (8192, 128), (8192, 16), (3000, 256)])
def test_align_large_matches_oracle(T, bm):
    rng = np.random.default_rng(T * 31 + bm)
    # zipf-like popularity to exercise empty and huge experts
    p = 1.0 / np.arange(1, 257) ** 1.1
    p /= p.sum()
    ids = np.stack([rng.choice(256, 8, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    s, e, total = run_align(ids, bm)
    rs, re_, rn = O.moe_align_block_size(ids, bm, 256)
    assert total == int(rn[0])
    assert np.array_equal(s, rs)
    assert np.array_equal(e, re_)


def test_align_rejects_bad_expert_ids():
    t = torch.tensor([[0, 300]], dtype=torch.int32, device=DEV)
    s = torch.empty(64, dtype=torch.int32, device=DEV)
    e = torch.empty(4, dtype=torch.int32, device=DEV)
    ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_align(t, 256, 16, s, e, ntp)
    torch.cuda.synchronize()
    assert ops.read_status() & ops.ERR_BAD_EXPERT


def test_permute_rows():
    T, K, H, bm = 50, 8, 6144, 16
    rng = np.random.default_rng(3)
    ids = np.stack([rng.choice(256, K, replace=False) for _ in range(T)]).astype(np.int32)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    rs, _, rn = O.moe_align_block_size(ids, bm, 256)
    s = torch.from_numpy(rs).to(DEV)
    ntp = torch.from_numpy(rn).to(DEV)
    dst = torch.full((rs.size + 16, H), 7.0, dtype=torch.bfloat16, device=DEV)
    ops.permute_rows(x, s, ntp, K, T * K, dst, max_rows=dst.shape[0])
    finish()
    xs = x.cpu()
    for p, v in enumerate(rs):
        row = dst[p].cpu()
        if v < T * K:
            assert torch.equal(row, xs[v // K])
        else:
            pass  # dispatch pad: left untouched
    assert torch.all(dst[rs.size:].cpu() == 7.0)  # rows past ntp untouched


@pytest.mark.parametrize("T,bm", [(50, 16), (8192, 256)])  # one-CTA and multi-launch paths
def test_align_pos_of_inverts_sorted_ids(T, bm):
    """pos_of[i] is the dispatch position of pair i: sorted_ids[pos_of[i]] == i, and
    the layout itself is the oracle's bit for bit."""
    K, E = 8, 256
    rng = np.random.default_rng(5 + T)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    rs, re, rn = O.moe_align_block_size(ids, bm, E)
    t = torch.from_numpy(ids).to(DEV)
    s = torch.empty(rs.size, dtype=torch.int32, device=DEV)
    e = torch.empty(re.size, dtype=torch.int32, device=DEV)
    ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
    pos = torch.full((T * K,), -1, dtype=torch.int32, device=DEV)
    ops.moe_align(t, E, bm, s, e, ntp, pos_of=pos)
    finish()
    assert np.array_equal(s.cpu().numpy(), rs) and np.array_equal(e.cpu().numpy(), re)
    p = pos.cpu().numpy()
    assert np.array_equal(rs[p], np.arange(T * K))


def balanced_layout_np(ids: np.ndarray, bm: int, E: int):
    """CPU statement of FUS_ALIGN_BALANCED: the reference's padded regions, each
    expert's c pairs spread over its nb = ceil(c/bm) blocks, ceil(c/nb) per block."""
    s_ref, e_ref, n_ref = O.moe_align_block_size(ids, bm, E)
    flat = ids.reshape(-1)
    numel = flat.size
    out = np.full_like(s_ref, numel)
    order = np.argsort(flat, kind="stable")
    counts = np.bincount(flat, minlength=E)
    start, src = 0, 0
    for e in range(E):
        c = int(counts[e])
        padded = -(-c // bm) * bm
        if c:
            nb = padded // bm
            pb = -(-c // nb)
            for q in range(c):
                out[start + (q // pb) * bm + q % pb] = order[src + q]
        start += padded
        src += c
    return out, e_ref, n_ref


@pytest.mark.parametrize("T,bm,skew", [(60, 64, False), (8192, 256, False), (8192, 256, True),
                                       (3000, 128, True)])
def test_align_balanced_layout(T, bm, skew):
    """FUS_ALIGN_BALANCED: same padded regions / expert ids / ntp as the reference
    layout, pairs spread evenly over each expert's blocks, pos_of its inverse."""
    K, E = 8, 256
    rng = np.random.default_rng(17 + T + bm)
    if skew:  # a few hot experts with several blocks each
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        ids = np.stack([rng.choice(E, K, replace=False, p=p / p.sum()) for _ in range(T)])
    else:
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
    ids = ids.astype(np.int32)
    rs, re, rn = balanced_layout_np(ids, bm, E)
    t = torch.from_numpy(ids).to(DEV)
    s = torch.empty(rs.size, dtype=torch.int32, device=DEV)
    e = torch.empty(re.size, dtype=torch.int32, device=DEV)
    ntp = torch.zeros(1, dtype=torch.int32, device=DEV)
    pos = torch.full((T * K,), -1, dtype=torch.int32, device=DEV)
    ops.moe_align(t, E, bm, s, e, ntp, pos_of=pos, flags=ops.ALIGN_BALANCED)
    finish()
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(e.cpu().numpy(), re) and int(ntp.item()) == int(rn[0])
    assert np.array_equal(rs[pos.cpu().numpy()], np.arange(T * K))
