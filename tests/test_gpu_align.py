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
