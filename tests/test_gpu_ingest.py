"""Checkpoint ingest on the GPU: FP8 (e4m3, 128 x 128 block scales) dequantisation
bit-exact against the oracle, and a Hugging Face layer (bf16 and FP8) loaded through
fusion_b200.ingest giving the same block output as the block built from the same
weights directly."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from fusion_b200 import ingest, ops, synth
from fusion_b200.block import MoEBlock
from gpu_util import DEV, finish, to_np
from oracle import reference_np as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(256, 384), (200, 136), (4096, 6144)])
def test_fp8_block_dequant_bit_exact(shape):
    rng = np.random.default_rng(shape[0])
    w = rng.standard_normal(shape).astype(np.float32) * 0.03
    q, s = ingest.fp8_quantize_blocks(w)
    out = torch.empty(shape, dtype=torch.bfloat16, device=DEV)
    ops.fp8_block_dequant(q.to(DEV), torch.from_numpy(s).to(DEV), out)
    finish()
    ref = O.fp8_block_dequant(q.view(torch.uint8).numpy(), s)
    assert np.array_equal(to_np(out), ref)


@pytest.mark.parametrize("fp8", [False, True])
def test_hf_layer_runs_like_direct_weights(tmp_path, fp8):
    d = synth.Dims(H=512, I=256, E=128, topk=8)
    L, seed = 5, 21
    w = synth.make_block_weights(seed, d, "cpu")
    k = ingest.layer_keys(L, d.E)
    sd = {k["gamma"]: w["gamma"], k["gate_w"]: w["gate_w"], k["bias"]: w["bias"]}

    def put(name, t):
        if fp8:
            q, s = ingest.fp8_quantize_blocks(t.float().numpy())
            sd[name], sd[name + "_scale_inv"] = q, torch.from_numpy(s)
        else:
            sd[name] = t

    for e in range(d.E):
        put(k[f"e{e}.gate"], w["w13"][e, :d.I])
        put(k[f"e{e}.up"], w["w13"][e, d.I:])
        put(k[f"e{e}.down"], w["w2"][e])
    put(k["s.gate"], w["w13s"][:d.I])
    put(k["s.up"], w["w13s"][d.I:])
    put(k["s.down"], w["w2s"])
    p = tmp_path / "ckpt.safetensors"
    ingest.write_safetensors(p, sd)
    got = ingest.load_moe_layer(ingest.read_safetensors(p), L, E=d.E, H=d.H, I=d.I, device=DEV)
    if fp8:  # the weights the checkpoint really holds: the oracle's dequantisation
        def deq(name):
            return torch.from_numpy(O.fp8_block_dequant(sd[name].view(torch.uint8).numpy(),
                                                        sd[name + "_scale_inv"].numpy()))
        ref_w = dict(w)
        ref_w["w13"] = torch.stack([torch.cat([deq(k[f"e{e}.gate"]), deq(k[f"e{e}.up"])])
                                    for e in range(d.E)]).to(torch.bfloat16)
        ref_w["w2"] = torch.stack([deq(k[f"e{e}.down"]) for e in range(d.E)]).to(torch.bfloat16)
        ref_w["w13s"] = torch.cat([deq(k["s.gate"]), deq(k["s.up"])]).to(torch.bfloat16)
        ref_w["w2s"] = deq(k["s.down"]).to(torch.bfloat16)
    else:
        ref_w = w
    for name in ("w13", "w2", "w13s", "w2s", "gamma"):
        assert torch.equal(got[name].cpu(), ref_w[name]), name
    ref_w = {n: t.to(DEV) for n, t in ref_w.items()}
    h, r = synth.make_inputs(seed, 3, d, DEV)
    a = MoEBlock(got["gamma"], got["gate_w"], got["bias"], got["w13"], got["w2"], got["w13s"],
                 got["w2s"])(h, r)
    b = MoEBlock(ref_w["gamma"], ref_w["gate_w"], ref_w["bias"], ref_w["w13"], ref_w["w2"],
                 ref_w["w13s"], ref_w["w2s"])(h, r)
    finish()
    assert torch.equal(a.out.view(torch.int16), b.out.view(torch.int16))
    assert torch.equal(a.topi, b.topi)
