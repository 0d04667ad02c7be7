"""CPU checks of the C-ABI library: it loads, exports every declared symbol, rejects
bad arguments on the host, and its host-side generator is deterministic."""

from __future__ import annotations

import ctypes
import re

import numpy as np
import torch

from conftest import ROOT
from fusion_b200 import _lib as L
from fusion_b200 import synth


def _declared() -> list[str]:
    text = (ROOT / "include" / "fusion_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fus_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert set(L.SIGNATURES) == set(names)
    assert lib.fus_version() >= 1


def test_host_argument_validation():
    lib = L.lib()
    # N not a multiple of 8
    rc = lib.fus_add_rmsnorm(None, 0, None, 0, None, None, 0, None, 0, 4, 7, 1e-5, 1, 1, None, None)
    assert rc == -1 and "multiple of 8" in L.last_error()
    # bad block_n for the GEMM is rejected before any launch
    g = (L.GemmGroup * 1)()
    rc = lib.fus_grouped_gemm(g, 1, 128, 64, 1, 0, 16, 1, 0, None, None)
    assert rc == -1  # null pointers
    rc = lib.fus_grouped_gemm(g, 3, 128, 64, 1, 0, 16, 1, 0, None, None)
    assert rc == -1
    rc = lib.fus_router_topk(None, 1, None, None, None, None, 4, 256, 8, 2.5, 1, None, None)
    assert rc == -1
    rc = lib.fus_moe_align(None, 8, 256, 16, None, 0, None, 0, None, None, 0, None, None)
    assert rc == -1


def test_router_nsplit_is_normalised():
    for T in (1, 2, 7, 32, 256, 2048, 8192):
        for planes in (1, 3):
            n = L.lib().fus_router_nsplit(T, 6144, 256, planes)
            ks = planes * 6144 // 64
            kps = -(-ks // n)
            assert n >= 1 and -(-ks // kps) == n


def test_block_workspace_grows_with_T():
    d = L.BlockDesc(H=6144, I=2048, E=256, topk=8, eps=1e-5, routed_scale=2.5, renorm=1,
                    nplanes=3)
    prev = 0
    for T in (1, 32, 256, 2048, 8192):
        bn = L.lib().fus_moe_block_pick_block_n(T, 256, 8)
        ws = L.lib().fus_moe_block_workspace(ctypes.byref(d), T, bn)
        assert ws > prev
        prev = ws


def _glm_desc(shared: bool, flags: int) -> L.BlockDesc:
    """A GLM-5.2 block descriptor with fake, 256-byte aligned weight addresses (host
    checks compare pointers with NULL and test alignment only; nothing is dereferenced)."""
    d = L.BlockDesc(H=6144, I=2048, E=256, topk=8, eps=1e-5, routed_scale=2.5, renorm=1,
                    nplanes=3, n_group=1, topk_group=1, flags=flags)
    for i, name in enumerate(("gamma", "wa", "w13", "w2")):
        setattr(d, name, ctypes.c_void_p(0x10000 * (i + 1)))
    d.bias = ctypes.c_void_p(0x90000)
    if shared:
        d.w13s = ctypes.c_void_p(0xA0000)
        d.w2s = ctypes.c_void_p(0xB0000)
    return d


def test_block_check_accepts_default_calls_at_every_size():
    """The block's pre-launch checks pass for the default descriptor at decode and
    prefill sizes, with and without the shared expert: a decode call whose front end
    would reject its own arguments fails here, on the CPU."""
    lib = L.lib()
    for shared in (True, False):
        d = _glm_desc(shared, 0)
        for T in (1, 2, 8, 16, 17, 32, 256, 2048, 8192):
            bn = lib.fus_moe_block_pick_block_n(T, 256, 8)
            ws = lib.fus_moe_block_workspace(ctypes.byref(d), T, bn)
            rc = lib.fus_moe_block_check(ctypes.byref(d), T, 0, ws)
            assert rc == 0, (shared, T, L.last_error())


def test_block_check_rejects_bad_arguments():
    lib = L.lib()
    d = _glm_desc(True, 0)
    ws = lib.fus_moe_block_workspace(ctypes.byref(d), 1, 0)
    assert lib.fus_moe_block_check(ctypes.byref(d), 1, 0, ws - 1) == -1
    assert "workspace" in L.last_error()
    d.w2s = None  # shared gate-up without shared down
    assert lib.fus_moe_block_check(ctypes.byref(d), 1, 0, ws) == -1
    assert "missing weights" in L.last_error()
    d = _glm_desc(True, 1)  # the flags field is reserved
    assert lib.fus_moe_block_check(ctypes.byref(d), 1, 0, ws) == -1
    assert "flags" in L.last_error()
    d = _glm_desc(True, 0)
    d.topk = 40  # 40 slots per token: past the decode front end's limit
    assert lib.fus_moe_block_check(ctypes.byref(d), 4, 16, 1 << 40) != 0
    assert lib.fus_moe_block_check(ctypes.byref(_glm_desc(True, 0)), 0, 0, 0) == 0


def test_synth_host_deterministic_and_sliceable():
    a = synth.make("w13", (4, 64, 96), 5)
    b = synth.make("w13", (4, 64, 96), 5)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    # expert 2 regenerated alone equals the slice of the stack
    n = 64 * 96
    c = synth.make("w13", (64, 96), 5, offset=2 * n)
    assert torch.equal(a[2].view(torch.int16), c.view(torch.int16))
    z = synth.make("h", (1 << 20,), 9).float().numpy()
    assert abs(z.mean()) < 5e-3 and abs(z.std() - 1.0) < 5e-3
    g = synth.make("gamma", (4096,), 9).float().numpy()
    assert abs(g.mean() - 1.0) < 2e-3 and abs(g.std() - 0.02) < 2e-3
    f = synth.make("gate_w", (4096,), 9).numpy()
    assert f.dtype == np.float32 and abs(f.std() - 0.02) < 2e-3


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    """No fallback: without the built library every entry point raises."""
    import pytest

    from fusion_b200 import _lib as L

    monkeypatch.setattr(L, "_lib", None)
    monkeypatch.setattr(L, "LIB_PATH", tmp_path / "libfusion_b200.so")
    with pytest.raises(RuntimeError, match="not built"):
        L.lib()
    with pytest.raises(RuntimeError, match="not built"):
        L.call("fus_version")
