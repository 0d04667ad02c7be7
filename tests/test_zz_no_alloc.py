"""The allocation-free dispatch-layout entry point (fus_moe_align_noalloc).

Some callers cannot allocate device memory: serving engines whose pool owns nearly all of
HBM from start-up, and loops that cannot afford cudaMalloc's device synchronisation.
For them the library keeps moe_align's scratch in a fixed device array. These tests call
that entry point through the C ABI and require the same layout, bit for bit, as the
workspace-taking fus_moe_align, on two calls in a row (the second call must not be
disturbed by what the first left in the shared scratch).

This file is named to be collected last, so a run that stops at the first failure has
already run every other test."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusion_b200 import _lib as L
from fusion_b200 import ops

E, K = 256, 8


def _ids(T: int, seed: int) -> torch.Tensor:
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, E + 1) ** 1.1
    p /= p.sum()
    ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    return torch.from_numpy(ids).cuda()


def _buffers(numel: int, bm: int):
    cap = (numel + E * (bm - 1) + bm - 1) // bm * bm
    s = torch.full((cap,), -7, dtype=torch.int32, device="cuda")
    e = torch.full((cap // bm,), -7, dtype=torch.int32, device="cuda")
    n = torch.zeros(1, dtype=torch.int32, device="cuda")
    return s, e, n


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = L.lib()
    stream = torch.cuda.current_stream().cuda_stream
    status = ops.status_tensor()
    # the largest accepted input (uses the scratch), then a smaller one on the same scratch
    for T, bm, seed in ((8192, 128, 1), (3000, 16, 2)):
        ids = _ids(T, seed)
        numel = ids.numel()
        s0, e0, n0 = _buffers(numel, bm)
        ops.moe_align(ids, E, bm, s0, e0, n0)  # reference: caller-provided workspace
        s1, e1, n1 = _buffers(numel, bm)
        rc = lib.fus_moe_align_noalloc(ids.data_ptr(), numel, E, bm, s1.data_ptr(), s1.numel(),
                                       e1.data_ptr(), e1.numel(), n1.data_ptr(), stream,
                                       status.data_ptr())
        assert rc == 0, L.last_error()
        torch.cuda.synchronize()
        ops.check_status()
        total = int(n0.item())
        assert int(n1.item()) == total
        assert torch.equal(s1[:total], s0[:total])
        assert torch.equal(e1[: total // bm], e0[: total // bm])


def test_noalloc_rejects_inputs_beyond_its_scratch():
    rc = L.lib().fus_moe_align_noalloc(None, 65537, E, 16, None, 0, None, 0, None, None, None)
    assert rc == -3 and "65536" in L.last_error()
