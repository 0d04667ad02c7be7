"""Checkpoint ingest on the host: the .safetensors reader/writer, the Hugging Face key
map into sglang's FusedMoE layout (gate rows then up rows in w13), and the e4m3 decode
of the oracle against torch's float8_e4m3fn."""

from __future__ import annotations

import numpy as np
import torch

from fusion_b200 import ingest
from oracle import reference_np as O


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    ts = {
        "a.bf16": torch.randn(3, 5, generator=g).to(torch.bfloat16),
        "b.f32": torch.randn(7, generator=g),
        "c.fp8": (torch.randn(4, 16, generator=g) * 3).to(torch.float8_e4m3fn),
        "d.i32": torch.arange(6, dtype=torch.int32).view(2, 3),
        "e.empty": torch.empty(0, 4, dtype=torch.bfloat16),
    }
    p = tmp_path / "x.safetensors"
    ingest.write_safetensors(p, ts)
    back = ingest.read_safetensors(p)
    assert set(back) == set(ts)
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape
        assert torch.equal(back[k].view(torch.uint8), v.view(torch.uint8))
    only = ingest.read_safetensors(p, names={"b.f32"})
    assert list(only) == ["b.f32"]


def _hf_layer(L, E, H, I, seed, shared=True):
    g = torch.Generator().manual_seed(seed)
    k = ingest.layer_keys(L, E, shared)
    sd = {k["gamma"]: torch.randn(H, generator=g).to(torch.bfloat16),
          k["gate_w"]: torch.randn(E, H, generator=g),
          k["bias"]: torch.randn(E, generator=g)}
    for e in range(E):
        sd[k[f"e{e}.gate"]] = torch.randn(I, H, generator=g).to(torch.bfloat16)
        sd[k[f"e{e}.up"]] = torch.randn(I, H, generator=g).to(torch.bfloat16)
        sd[k[f"e{e}.down"]] = torch.randn(H, I, generator=g).to(torch.bfloat16)
    if shared:
        for part, shape in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
            sd[k[f"s.{part}"]] = torch.randn(*shape, generator=g).to(torch.bfloat16)
    return sd, k


def test_hf_layer_into_fused_moe_layout(tmp_path):
    L, E, H, I = 3, 6, 64, 32
    sd, k = _hf_layer(L, E, H, I, 1)
    p = tmp_path / "layer.safetensors"
    ingest.write_safetensors(p, sd)
    w = ingest.load_moe_layer(ingest.read_safetensors(p), L, E=E, H=H, I=I, device="cpu")
    assert w["w13"].shape == (E, 2 * I, H) and w["w2"].shape == (E, H, I)
    for e in range(E):
        assert torch.equal(w["w13"][e, :I], sd[k[f"e{e}.gate"]])  # gate rows first
        assert torch.equal(w["w13"][e, I:], sd[k[f"e{e}.up"]])
        assert torch.equal(w["w2"][e], sd[k[f"e{e}.down"]])
    assert torch.equal(w["w13s"][:I], sd[k["s.gate"]]) and torch.equal(w["w13s"][I:], sd[k["s.up"]])
    assert torch.equal(w["w2s"], sd[k["s.down"]])
    assert w["gate_w"].dtype == torch.float32 and torch.equal(w["gate_w"], sd[k["gate_w"]])
    assert torch.equal(w["gamma"], sd[k["gamma"]])


def test_e4m3_decode_matches_torch():
    bits = np.arange(256, dtype=np.uint8)
    ours = O.e4m3_to_f32(bits)
    ref = torch.from_numpy(bits).view(torch.float8_e4m3fn).float().numpy()
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan], ref[~nan])


def test_fp8_quantize_round_trip_is_close():
    rng = np.random.default_rng(2)
    w = rng.standard_normal((256, 384)).astype(np.float32) * 0.02
    q, s = ingest.fp8_quantize_blocks(w)
    back = O.fp8_block_dequant(q.view(torch.uint8).numpy(), s)
    assert s.shape == (2, 3)
    assert float(np.abs(back - w).max()) <= 0.07 * float(np.abs(w).max())  # e4m3: 3-bit mantissa
